// ggml_blocks.cuh -- GGML block geometry and exact per-unit decoders (device).
//
// Type ids and (block_size, bytes_per_block) follow the GGML enum as listed in
// pyrite/ggml_types.py:34-73; the 21 decodable ids are the ones of the
// reference's native table (pyrite/kernels/native.c:451-473).
//
// A "unit" is 32 consecutive values of one block (a whole block for the
// 32-value formats, one of eight for the 256-value super-blocks, 32 scalars for
// the one-value formats).  decode_unit<T> produces those values in precision T:
//   * T = double reproduces the reference's arithmetic exactly (every product
//     there is exact in double, pyrite/kernels/native.c:129-437);
//   * T = float gives, for every type, the correctly rounded fp32 value of the
//     reference's double: all scale products are exact in fp32 and the single
//     rounding happens in the last add/fma.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace pyr {

enum GgmlType : int {
  F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
  Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, IQ4_NL = 20, IQ4_XS = 23,
  I8 = 24, I16 = 25, I32 = 26, I64 = 27, F64 = 28, BF16 = 30,
};

struct TypeGeo { int id; int bs; int bpb; };

// Same order as the reference table so pyrite_native_types() reports the
// same sequence (pyrite/kernels/native.c:451-473).
constexpr TypeGeo kTypes[] = {
  {F32, 1, 4},     {F16, 1, 2},     {Q4_0, 32, 18},   {Q4_1, 32, 20},  {Q5_0, 32, 22},
  {Q5_1, 32, 24},  {Q8_0, 32, 34},  {Q8_1, 32, 36},   {Q2_K, 256, 84}, {Q3_K, 256, 110},
  {Q4_K, 256, 144}, {Q5_K, 256, 176}, {Q6_K, 256, 210}, {IQ4_NL, 32, 18}, {IQ4_XS, 256, 136},
  {I8, 1, 1},      {I16, 1, 2},     {I32, 1, 4},      {I64, 1, 8},     {F64, 1, 8},
  {BF16, 1, 2},
};
constexpr int kNumTypes = sizeof(kTypes) / sizeof(kTypes[0]);

template <int TY> struct Geo;
#define PYR_GEO(T, B, P) template <> struct Geo<T> { static constexpr int bs = B, bpb = P; };
PYR_GEO(F32, 1, 4) PYR_GEO(F16, 1, 2) PYR_GEO(Q4_0, 32, 18) PYR_GEO(Q4_1, 32, 20)
PYR_GEO(Q5_0, 32, 22) PYR_GEO(Q5_1, 32, 24) PYR_GEO(Q8_0, 32, 34) PYR_GEO(Q8_1, 32, 36)
PYR_GEO(Q2_K, 256, 84) PYR_GEO(Q3_K, 256, 110) PYR_GEO(Q4_K, 256, 144) PYR_GEO(Q5_K, 256, 176)
PYR_GEO(Q6_K, 256, 210) PYR_GEO(IQ4_NL, 32, 18) PYR_GEO(IQ4_XS, 256, 136) PYR_GEO(I8, 1, 1)
PYR_GEO(I16, 1, 2) PYR_GEO(I32, 1, 4) PYR_GEO(I64, 1, 8) PYR_GEO(F64, 1, 8) PYR_GEO(BF16, 1, 2)
#undef PYR_GEO

// Expand F(TYPE) over every decodable type (kernel instantiation / dispatch).
#define PYR_FOR_EACH_TYPE(F) \
  F(F32) F(F16) F(Q4_0) F(Q4_1) F(Q5_0) F(Q5_1) F(Q8_0) F(Q8_1) F(Q2_K) F(Q3_K) F(Q4_K) \
  F(Q5_K) F(Q6_K) F(IQ4_NL) F(IQ4_XS) F(I8) F(I16) F(I32) F(I64) F(F64) F(BF16)

inline const TypeGeo* find_type(int id) {
  for (int i = 0; i < kNumTypes; ++i)
    if (kTypes[i].id == id) return &kTypes[i];
  return nullptr;
}

// The IQ4_NL / IQ4_XS non-linear 4-bit code book (pyrite/tensor_ops.py:205-207).
__device__ __constant__ const int8_t kIq4Book[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                                     1,    13,   25,  38,  53,  69,  89,  113};

__device__ __forceinline__ unsigned ld_u8(const uint8_t* p) { return *p; }
__device__ __forceinline__ unsigned ld_u16(const uint8_t* p) { return (unsigned)p[0] | ((unsigned)p[1] << 8); }
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

template <typename T> __device__ __forceinline__ T half_val(unsigned h) {
  return (T)__half2float(__ushort_as_half((unsigned short)h));
}

// 6-bit (scale, min) pair j of the 12-byte K-quant scale field
// (pyrite/kernels/native.c:52-60).
__device__ __forceinline__ void k4_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Scalar formats: value i of a one-value "block".
template <int TY, typename T> __device__ __forceinline__ T scalar_val(const uint8_t* p) {
  if constexpr (TY == F32) { return (T)__uint_as_float(ld_u32(p)); }
  else if constexpr (TY == F16) { return half_val<T>(ld_u16(p)); }
  else if constexpr (TY == BF16) { return (T)__uint_as_float(ld_u16(p) << 16); }
  else if constexpr (TY == I8) { return (T)(int8_t)ld_u8(p); }
  else if constexpr (TY == I16) { return (T)(int16_t)ld_u16(p); }
  else if constexpr (TY == I32) { return (T)(int32_t)ld_u32(p); }
  else if constexpr (TY == I64) {
    const long long v = (long long)((uint64_t)ld_u32(p) | ((uint64_t)ld_u32(p + 4) << 32));
    // via double, so the fp32 result is (float)(reference double)
    return (T)__ll2double_rn(v);
  } else {  // F64
    const unsigned long long b = (uint64_t)ld_u32(p) | ((uint64_t)ld_u32(p + 4) << 32);
    return (T)__longlong_as_double((long long)b);
  }
}

// Decode unit u (values 32u .. 32u+31 of the block starting at b) into v.
// Block formats only (bs >= 32).  Formulas restate pyrite/tensor_ops.py:90-448.
template <int TY, typename T>
__device__ __forceinline__ void decode_unit(const uint8_t* b, int u, T (&v)[32]) {
  if constexpr (TY == Q4_0) {
    const T d = half_val<T>(ld_u16(b));
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = d * (T)((int)(b[2 + i] & 15) - 8);
      v[16 + i] = d * (T)((int)(b[2 + i] >> 4) - 8);
    }
  } else if constexpr (TY == Q4_1) {
    const T d = half_val<T>(ld_u16(b)), m = half_val<T>(ld_u16(b + 2));
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = d * (T)(b[4 + i] & 15) + m;
      v[16 + i] = d * (T)(b[4 + i] >> 4) + m;
    }
  } else if constexpr (TY == Q5_0) {
    const T d = half_val<T>(ld_u16(b));
    const uint32_t qh = ld_u32(b + 2);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int lo = (b[6 + i] & 15) | (int)(((qh >> i) & 1u) << 4);
      const int hi = (b[6 + i] >> 4) | (int)(((qh >> (16 + i)) & 1u) << 4);
      v[i] = d * (T)(lo - 16);
      v[16 + i] = d * (T)(hi - 16);
    }
  } else if constexpr (TY == Q5_1) {
    const T d = half_val<T>(ld_u16(b)), m = half_val<T>(ld_u16(b + 2));
    const uint32_t qh = ld_u32(b + 4);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int lo = (b[8 + i] & 15) | (int)(((qh >> i) & 1u) << 4);
      const int hi = (b[8 + i] >> 4) | (int)(((qh >> (16 + i)) & 1u) << 4);
      v[i] = d * (T)lo + m;
      v[16 + i] = d * (T)hi + m;
    }
  } else if constexpr (TY == Q8_0 || TY == Q8_1) {
    const T d = half_val<T>(ld_u16(b));
    const uint8_t* qs = b + (TY == Q8_0 ? 2 : 4);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = d * (T)(int8_t)qs[i];
  } else if constexpr (TY == IQ4_NL) {
    const T d = half_val<T>(ld_u16(b));
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = d * (T)kIq4Book[b[2 + i] & 15];
      v[16 + i] = d * (T)kIq4Book[b[2 + i] >> 4];
    }
  } else if constexpr (TY == IQ4_XS) {
    const T d = half_val<T>(ld_u16(b));
    const unsigned sh = ld_u16(b + 2);
    const int ls = ((b[4 + u / 2] >> (4 * (u & 1))) & 15) | (int)(((sh >> (2 * u)) & 3u) << 4);
    const T dl = d * (T)(ls - 32);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const unsigned q = b[8 + 16 * u + i];
      v[i] = dl * (T)kIq4Book[q & 15];
      v[16 + i] = dl * (T)kIq4Book[q >> 4];
    }
  } else if constexpr (TY == Q2_K) {
    const T d = half_val<T>(ld_u16(b + 80)), dmin = half_val<T>(ld_u16(b + 82));
    const int h = u >> 2, g = u & 3;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int sc = b[8 * h + 2 * g + (l >> 4)];
      const int q = (b[16 + 32 * h + l] >> (2 * g)) & 3;
      v[l] = (d * (T)(sc & 15)) * (T)q - dmin * (T)(sc >> 4);
    }
  } else if constexpr (TY == Q3_K) {
    const T d = half_val<T>(ld_u16(b + 108));
    const int h = u >> 2, g = u & 3;
    T dl[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int k = 8 * h + 2 * g + s;
      const int low = (k < 8) ? (b[96 + k] & 15) : (b[96 + k - 8] >> 4);
      const int high = (b[104 + (k & 3)] >> (2 * (k >> 2))) & 3;
      dl[s] = d * (T)((low | (high << 4)) - 32);
    }
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int q = ((b[32 + 32 * h + l] >> (2 * g)) & 3) - (((b[l] >> (4 * h + g)) & 1) ? 0 : 4);
      v[l] = dl[l >> 4] * (T)q;
    }
  } else if constexpr (TY == Q4_K || TY == Q5_K) {
    const T d = half_val<T>(ld_u16(b)), dmin = half_val<T>(ld_u16(b + 2));
    const int p = u >> 1, hi = u & 1;
    int sc, mn;
    k4_scale_min(b + 4, u, sc, mn);
    const T d1 = d * (T)sc, m1 = dmin * (T)mn;
    const uint8_t* qs = b + (TY == Q4_K ? 16 : 48) + 32 * p;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      int q = hi ? (qs[l] >> 4) : (qs[l] & 15);
      if constexpr (TY == Q5_K) q += ((b[16 + l] >> u) & 1) ? 16 : 0;
      v[l] = d1 * (T)q - m1;
    }
  } else if constexpr (TY == Q6_K) {
    const T d = half_val<T>(ld_u16(b + 208));
    const int h = u >> 2, t = u & 3;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const unsigned lq = b[64 * h + 32 * (t & 1) + l];
      const int low = (t >= 2) ? (int)(lq >> 4) : (int)(lq & 15);
      const int high = (b[128 + 32 * h + l] >> (2 * t)) & 3;
      const int sc = (int8_t)b[192 + 8 * h + 2 * t + (l >> 4)];
      v[l] = d * (T)sc * (T)((low | (high << 4)) - 32);
    }
  }
}

}  // namespace pyr

/*
 * pyrite_b200.h -- C ABI of libpyrite_b200.so, the B200 implementation of
 * Pyrite's fused GGML dequantize x matrix-vector kernel library.
 *
 * Section 1 is a drop-in for the reference's C kernel library
 * (pyrite/kernels/native.c, bound by ctypes in pyrite/kernels/native.py:
 * 126-147): same symbol names, signatures, argument meaning and return codes.
 * Section 2 is the device-resident path used by the B200 runtime.
 *
 * All entry points are plain C: pointers, sizes and an opaque stream handle.
 * Return codes: 0 on success, negative on error (see PYRITE_E_*).
 */
#ifndef PYRITE_B200_H
#define PYRITE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes.  -1..-3 are the reference's (pyrite/kernels/native.c:496-525);
 * -4 is new: the CUDA runtime reported an error (no device, launch failure). */
#define PYRITE_E_TYPE (-1)   /* unknown / non-decodable GGML type id          */
#define PYRITE_E_SHAPE (-2)  /* rows or cols zero, cols not block aligned,
                                or the byte size overflows                    */
#define PYRITE_E_BUFFER (-3) /* NULL pointer, or data_len != rows * row_bytes */
#define PYRITE_E_CUDA (-4)   /* CUDA error                                    */

/* ---- 1. Reference-compatible entry points (host buffers, fp64) ---------- */

/* Replaces pyrite_native_types (pyrite/kernels/native.c:484-494).
 * ids == NULL: returns the number of supported GGML type ids.  Otherwise
 * writes up to `capacity` ids and returns how many were written.  The set is
 * the reference's 21 decodable types, in the reference's order. */
int pyrite_native_types(int *ids, size_t capacity);

/* Replaces pyrite_matvec (pyrite/kernels/native.c:518-555).
 * out[r] = sum_c W[r, c] * x[c] for `rows` consecutive rows of a GGML matrix
 * whose payload (`data`, `data_len` bytes, host memory, borrowed for the call)
 * holds rows of cols/block_size blocks each.  x has `cols` doubles, out has
 * `rows`.  Runs on the current CUDA device, decoding and accumulating in fp64;
 * blocks until `out` is written. */
int pyrite_matvec(int type_id, const uint8_t *data, size_t data_len, const double *x,
                  double *out, size_t rows, size_t cols);

/* Replaces pyrite_dequantize_rows (pyrite/kernels/native.c:557-576).
 * Writes rows x cols doubles (row-major) decoded from the payload.  Values are
 * identical to the reference's. */
int pyrite_dequantize_rows(int type_id, const uint8_t *data, size_t data_len, double *out,
                           size_t rows, size_t cols);

/* ---- 2. Device-resident path (new; no reference counterpart) ------------- */

/* Geometry of a type: values per block and bytes per block (the reference
 * keeps this table in pyrite/ggml_types.py:34-73). */
int pyrite_type_geometry(int type_id, size_t *block_size, size_t *bytes_per_block);

/* Flags of pyrite_cuda_matvec. */
#define PYRITE_F_STATIC_WEIGHTS 1u /* the payload is not written by the kernel that precedes
                                      this call in the stream: its HBM stream may start
                                      before that kernel finishes (programmatic dependent
                                      launch); x and y are still ordered after it */
#define PYRITE_F_ACCUMULATE 2u     /* pyrite_cuda_matvec / _prepared / _transformed:
                                      y += W x (a residual stream) instead of y = W x */

/* Operations a batch-1 matvec can run on its whole output y (rows values) in
 * the last of its CTAs to finish (pyrite_cuda_matvec_prepared_post): the glue
 * between the projections of a decode step without a launch of its own. */
#define PYRITE_POST_NONE 0
#define PYRITE_POST_RMSNORM_ENCODE 1  /* out = y * weight / sqrt(mean(y^2) + eps), fp64
                                         statistics (executor.py:621-624), encoded */
#define PYRITE_POST_SILU_MUL_ENCODE 2 /* y = [gate | up]: out = silu(gate) * up
                                         (dense.py:491-494), encoded */
#define PYRITE_POST_ARGMAX 3          /* tokens[*pos + 1] = first index of max(y) unless
                                         that position still holds the prompt; *pos += 1
                                         (sampler.py:12-15) */
typedef struct pyrite_post_op {
  int op;               /* PYRITE_POST_* */
  int prompt_len;       /* ARGMAX */
  int max_ctx;          /* ARGMAX: length of `tokens` */
  double eps;           /* RMSNORM_ENCODE */
  const float *weight;  /* RMSNORM_ENCODE: rows values */
  float *out;           /* RMSNORM_ENCODE (may be NULL) / SILU_MUL_ENCODE (rows/2 values) */
  void *workspace;      /* RMSNORM / SILU: the encoding of out (256-byte aligned, at least
                           pyrite_cuda_workspace_size(0, n, 1) bytes for n = len(out)) */
  size_t workspace_len;
  unsigned *ticket;     /* device counter, zero before the call and left zero by it; one per
                           call that can overlap another on the GPU */
  void *scratch;        /* ARGMAX: pyrite_cuda_post_scratch_size() bytes */
  size_t scratch_len;
  int *tokens;          /* ARGMAX */
  int *pos;             /* ARGMAX */
} pyrite_post_op;

/* The activation of a batch-1 matvec computed inside it (every CTA encodes
 * its own copy in shared memory) instead of by a kernel of its own: */
#define PYRITE_X_RMSNORM 1   /* x' = x * norm_weight / sqrt(mean(x^2) + eps), fp64 statistics */
#define PYRITE_X_SILU_MUL 2  /* x = [gate (cols) | up (cols)]: x' = silu(gate) * up */

/* y = W x' for the transformed activation x' above (executor.py:621-624 then
 * the projection; or dense.py:491-494 then the down projection).  x_out
 * receives x' in fp32 for later consumers.  Two forms, the same results up to
 * fp32 rounding: the batch-1 kernel's CTAs each compute x' in their prologue
 * (one launch), or the operation's own kernel writes x_out and `workspace`
 * (as for pyrite_cuda_matvec_prepared) and the product follows.  Given x_out
 * and a workspace, the library picks the faster form for the size; without
 * them only the prologue form exists (formats with the batch-1 kernel, vectors
 * 16-byte aligned).  flags: PYRITE_F_*. */
int pyrite_cuda_matvec_transformed(int type_id, const void *weights, size_t weights_len, const float *x,
                                   int x_op, const float *norm_weight, double eps, float *x_out,
                                   void *workspace, size_t workspace_len, float *y, size_t rows,
                                   size_t cols, unsigned flags, void *stream);

/* The form pyrite_cuda_matvec_transformed takes for these arguments given a
 * workspace: 1 = prologue (the workspace is left untouched), 0 = the
 * operation's own kernel first (afterwards the workspace and x_out hold x',
 * so further matrices on the same x' can use pyrite_cuda_matvec_prepared),
 * or a PYRITE_E_* code.  Host only; nothing is launched. */
int pyrite_cuda_matvec_transformed_form(int type_id, const void *weights, size_t weights_len, const float *x,
                                        int x_op, const float *norm_weight, const float *x_out, size_t rows,
                                        size_t cols);

/* Scratch bytes PYRITE_POST_ARGMAX needs on the current device. */
size_t pyrite_cuda_post_scratch_size(void);

/* pyrite_cuda_matvec_prepared followed by `post` on y, in one launch where the
 * batch-1 kernel takes the format (else the product and a separate kernel).
 * Same validation codes; a malformed `post` is PYRITE_E_BUFFER. */
int pyrite_cuda_matvec_prepared_post(int type_id, const void *weights, size_t weights_len,
                                     const float *x, const void *workspace, size_t workspace_len,
                                     float *y, size_t rows, size_t cols, unsigned flags,
                                     const pyrite_post_op *post, void *stream);

/* Device workspace bytes pyrite_cuda_matvec needs for `ncols` columns of
 * `cols` values (the activation is re-encoded there before the product). */
size_t pyrite_cuda_workspace_size(int type_id, size_t cols, size_t ncols);

/* y[c*ldy + r] = sum_k W[r, k] * x[c*ldx + k] for r < rows, c < ncols.
 * `weights` (weights_len == rows * row_bytes) , `x`, `y` and `workspace` are
 * device pointers; fp32 activations, fp32 outputs within 1e-4 of the exact
 * product relative to sum_k |W[r,k] x[k]|.  `workspace` (256-byte aligned, at
 * least pyrite_cuda_workspace_size bytes) holds the activation re-encoded as
 * int8 digits with per-32-value scales (three digits where a block holds
 * values far below its largest, e.g. an outlier channel); it must not be shared
 * by calls that overlap on the GPU.  Enqueued on `stream` (a cudaStream_t,
 * NULL = legacy default stream); returns without waiting.  Same validation
 * codes as pyrite_matvec.  This is the row-range call of the reference's
 * executor (pyrite/executor.py:481-509): pass the address of the first row of
 * the range and the range's row count.  `flags`: PYRITE_F_*. */
int pyrite_cuda_matvec(int type_id, const void *weights, size_t weights_len, const float *x,
                       long long ldx, float *y, long long ldy, size_t rows, size_t cols,
                       size_t ncols, unsigned flags, void *workspace, size_t workspace_len,
                       void *stream);

/* Re-encode x (ncols columns of `cols` values, cols a multiple of 32) into
 * `workspace` for pyrite_cuda_matvec_prepared: several matrices that share
 * one activation (Q/K/V, gate/up) then pay for the encoding once. */
int pyrite_cuda_prepare_x(const float *x, long long ldx, size_t cols, size_t ncols, void *workspace,
                          size_t workspace_len, void *stream);

/* y[r] = sum_k W[r, k] x[k] for one column whose encoding pyrite_cuda_prepare_x
 * wrote to `workspace` earlier on the same stream (x itself is still passed:
 * formats without an encoded-x kernel read it directly).  Same results and
 * codes as pyrite_cuda_matvec. */
int pyrite_cuda_matvec_prepared(int type_id, const void *weights, size_t weights_len, const float *x,
                                const void *workspace, size_t workspace_len, float *y, size_t rows,
                                size_t cols, unsigned flags, void *stream);

/* Largest `cols` pyrite_cuda_matvec_noalloc accepts.  Its fixed scratch array
 * (108 KiB per GPU) holds the encoding of up to 32768 values; wider
 * activations take the generic kernel, which reads x directly. */
#define PYRITE_NOALLOC_MAX_COLS 65536

/* No counterpart in the reference.  pyrite_cuda_matvec for one column, for
 * callers that cannot allocate device memory (a host runtime that owns all GPU
 * memory and forbids plugins to cudaMalloc, an allocation-free decode loop, an
 * FFI host with no device allocator): the activation's encoding goes to a
 * fixed array inside the library instead of a caller workspace, so this call
 * allocates nothing.  Same arguments (device pointers), results and codes as
 * pyrite_cuda_matvec with ncols = 1; cols above PYRITE_NOALLOC_MAX_COLS is
 * rejected with PYRITE_E_SHAPE before any GPU work.  The first call on each
 * device looks up the array's device address (cudaGetSymbolAddress) with that
 * device current -- make that first call before any stream capture.  The
 * address is kept for the life of the process: after cudaDeviceReset (or
 * anything else that destroys and re-creates the device's primary context)
 * it is stale, and this entry point must not be called again in that
 * process.  The one
 * array is shared by every call on a device and keeps the last call's bytes:
 * calls that may overlap on the GPU (different streams without ordering)
 * race on it; calls on one stream are ordered and safe. */
int pyrite_cuda_matvec_noalloc(int type_id, const void *weights, size_t weights_len, const float *x,
                               float *y, size_t rows, size_t cols, unsigned flags, void *stream);

/* out[r*cols + c] = W[r, c] as fp32 (the correctly rounded value of the
 * reference's fp64 result).  Device pointers; enqueued on `stream`. */
int pyrite_cuda_dequantize_rows(int type_id, const void *weights, size_t weights_len, float *out,
                                size_t rows, size_t cols, void *stream);

/* Number of visible CUDA devices (0 when there is no usable driver/device). */
int pyrite_cuda_device_count(void);

/* Device status word of the current device: bit 0 set when a kernel gave up
 * waiting for a copy (bounded waits never hang the GPU).  Synchronous read;
 * clears the word when `clear` is nonzero.  Returns the word or PYRITE_E_CUDA. */
int pyrite_cuda_status(int clear);

/* ---- 3. Quantizers (host; new) -------------------------------------------- */

/* Encode `count` values (a multiple of the block size) into GGML blocks at
 * `dst` (dst_len == count / block_size * bytes_per_block), using `threads`
 * host threads (<= 0: all).  Q8_0 / Q4_0 reproduce the reference's fixture
 * encoders byte for byte (scripts/build_vocab_fixture.py:54-92), Q2_K..Q6_K
 * its naive K-quant encoders (tests/k_quant.py:61-285); Q4_1 / Q5_0 / Q5_1
 * the gguf package's quantizers that the reference's tests use for those
 * formats (float32 arithmetic on float32-rounded inputs); IQ4_NL / IQ4_XS
 * are this library's own (the reference has no quantizer for them). */
int pyrite_quantize(int type_id, const double *src, size_t count, uint8_t *dst, size_t dst_len,
                    int threads);

/* Type ids pyrite_quantize accepts (ids == NULL: the count). */
int pyrite_quantize_types(int *ids, size_t capacity);

/* ---- 4. Decode-step glue (new; the reference runs these in Python fp64) -- */
/* Device pointers; every call only enqueues on `stream`.  The token id and
 * position are read from device memory (`tokens`, `pos`), so a whole decode
 * step can be captured in one CUDA graph and replayed without host syncs. */

/* out[0..cols) = row tokens[*pos] of a GGML `rows` x `cols` table
 * (executor.py:647-652, the embedding lookup). */
int pyrite_cuda_embed(int type_id, const void *table, size_t rows, size_t cols, const int *tokens,
                      const int *pos, float *out, void *stream);

/* out = x * w / sqrt(mean(x^2) + eps) (fp64 statistics, executor.py:621-624);
 * also writes its encoding for pyrite_cuda_matvec_prepared.  out may be NULL. */
int pyrite_cuda_rmsnorm_encode(const float *x, const float *weight, size_t n, double eps, float *out,
                               void *workspace, size_t workspace_len, void *stream);

/* qkv = [q (n_heads*128) | k (n_kv_heads*128) | v]: per-head RMSNorm of q and k
 * (norm weights may be NULL), NEOX RoPE with the fp64 (cos, sin) table row
 * *pos (rope_table: max_ctx x 64 double pairs), q to q_out, k and v appended
 * to the fp32 caches at row *pos (executor.py:700-731). */
int pyrite_cuda_qk_rope_kv(const float *qkv, const float *q_norm, const float *k_norm, int n_heads,
                           int n_kv_heads, int head_dim, double eps, const int *pos,
                           const void *rope_table, int max_ctx, float *q_out, float *k_cache,
                           float *v_cache, void *stream);

/* Grouped-query softmax attention of q over cache rows 0..*pos, scale
 * 1/sqrt(head_dim) (executor.py:733-755). */
int pyrite_cuda_attention(const float *q, const float *k_cache, const float *v_cache, const int *pos,
                          int n_heads, int n_kv_heads, int head_dim, int max_ctx, float *out,
                          void *stream);

/* pyrite_cuda_qk_rope_kv and pyrite_cuda_attention in one launch, the context
 * split over up to 32 CTAs per q head (flash-decoding: per-chunk max, sum and
 * weighted values, merged by the last CTA of the head), the output also
 * encoded into `workspace` for the output projection
 * (pyrite_cuda_matvec_prepared).  `scratch`: 16-byte aligned device memory of
 * pyrite_cuda_attention_scratch_size() bytes whose first n_heads words are
 * zero (the call leaves them zero); one per call that can overlap another. */
size_t pyrite_cuda_attention_scratch_size(int n_heads, int max_ctx);
int pyrite_cuda_attention_step(const float *qkv, const float *q_norm, const float *k_norm, int n_heads,
                               int n_kv_heads, int head_dim, double eps, const int *pos,
                               const void *rope_table, int max_ctx, float *k_cache, float *v_cache,
                               float *out, void *workspace, size_t workspace_len, void *scratch,
                               size_t scratch_len, void *stream);

/* act = silu(gate) * up for gate_up = [gate (f) | up (f)] (dense.py:491-494,
 * tensor_ops.py:509-510), also encoded for the down projection. */
int pyrite_cuda_silu_mul_encode(const float *gate_up, size_t f, float *act, void *workspace,
                                size_t workspace_len, void *stream);

/* Greedy sampling (sampler.py:12-15): the first index of the largest logit
 * is stored at tokens[*pos + 1] unless that position still holds the prompt
 * (*pos + 1 < prompt_len); then *pos += 1.  scratch: >= 1184 bytes. */
int pyrite_cuda_argmax_step(const float *logits, size_t n, void *scratch, size_t scratch_len,
                            int *tokens, int *pos, int prompt_len, int max_ctx, void *stream);

/* ---- several positions or sequences at once (prefill, multi-sequence decode)
 * The decode-step glue for `count` rows; each row's vector is a row of a
 * row-major array (`ld*` floats between rows) -- the layout of
 * pyrite_cuda_matvec's columns, so the projections of all rows run as one
 * multi-column (tensor-core) product.  The reference runs one position of one
 * sequence per forward pass (executor.py:878-939); each row here gets that
 * position's arithmetic.  Row j sits at position first + *pos + j * pos_step
 * (pos: device int, may be NULL = 0, read when the kernel runs so a CUDA graph
 * can replay the call): pos_step 1 = consecutive positions of one sequence
 * (batched prefill), pos_step 0 = one position shared by `count` sequences,
 * row j's KV cache cache_stride floats after row 0's (multi-sequence decode).
 * Rows outside [0, max_ctx) are rejected (host position) or skipped (device). */

/* out row j = table row ids[j * ids_stride + *pos] (ids, pos: device; pos may be NULL). */
int pyrite_cuda_embed_rows(int type_id, const void *table, size_t rows, size_t cols, const int *ids,
                           long long ids_stride, const int *pos, size_t count, float *out, long long ldo,
                           void *stream);
/* out row j = x row j * weight / sqrt(mean(x row j ^ 2) + eps), fp64 statistics. */
int pyrite_cuda_rmsnorm_rows(const float *x, long long ldx, const float *weight, size_t n, size_t count,
                             double eps, float *out, long long ldo, void *stream);
/* pyrite_cuda_qk_rope_kv for each row at its position: q rows to q_out, k and v
 * to that position's row of the row's caches. */
int pyrite_cuda_qk_rope_kv_rows(const float *qkv, long long ldqkv, const float *q_norm, const float *k_norm,
                                int n_heads, int n_kv_heads, int head_dim, double eps, int first, const int *pos,
                                int pos_step, long long cache_stride, int count, const void *rope_table,
                                int max_ctx, float *q_out, long long ldq, float *k_cache, float *v_cache,
                                void *stream);
/* Causal GQA attention: query row j (position p_j) over rows 0 .. p_j of its
 * cache, scale 1/sqrt(head_dim), fp32 (executor.py:733-755); the rows'
 * own k / v are written before (pyrite_cuda_qk_rope_kv_rows). */
int pyrite_cuda_attention_rows(const float *q, long long ldq, const float *k_cache, const float *v_cache,
                               long long cache_stride, int first, const int *pos, int pos_step, int count,
                               int n_heads, int n_kv_heads, int head_dim, int max_ctx, float *out, long long ldo,
                               void *stream);
/* Greedy token of each row of [count x n] logits (one sequence per row):
 * tokens[j * tok_stride + *pos + 1] = first index of the row's maximum unless
 * that position still holds the prompt (sampler.py:12-15).  *pos is left as it
 * is; pyrite_cuda_advance_pos adds 1 to it. */
int pyrite_cuda_argmax_rows(const float *logits, long long ld, size_t n, size_t count, int *tokens,
                            long long tok_stride, const int *pos, int prompt_len, int max_ctx, void *stream);
int pyrite_cuda_advance_pos(int *pos, void *stream);
/* act row j = silu(gate) * up for gate_up row j = [gate (f) | up (f)]. */
int pyrite_cuda_silu_mul_rows(const float *gate_up, long long ldgu, size_t f, size_t count, float *act,
                              long long lda, void *stream);

/* Greedy sampling over a vocabulary split across GPUs (each holds a contiguous
 * slice of the LM head's rows): pyrite_cuda_argmax_local reduces this GPU's
 * n logits to one 8-byte pair {float value, int32 id} with id = index_base +
 * the first index of the slice's largest logit (scratch as for
 * pyrite_cuda_argmax_step); after the pairs of all GPUs are exchanged (e.g.
 * an all-gather of 8 bytes per GPU), pyrite_cuda_argmax_pick takes the
 * largest value, the lowest id on ties -- sampler.py:12-15 over the whole
 * vocabulary -- and writes it like pyrite_cuda_argmax_step.  pair / pairs
 * 8-byte aligned device memory. */
int pyrite_cuda_argmax_local(const float *logits, size_t n, long long index_base, void *scratch,
                             size_t scratch_len, void *pair, void *stream);
int pyrite_cuda_argmax_pick(const void *pairs, size_t n_pairs, int *tokens, int *pos, int prompt_len,
                            int max_ctx, void *stream);

/* ---- routed experts (Qwen3-MoE feed-forward, executor.py:672-683, 757-793) ---- */

/* Router softmax (fp64) over n_experts logits, the top_k experts ordered by
 * (-probability, expert id), their weights renormalised to sum 1 when
 * norm_topk_prob, then multiplied by scale: expert_ids[top_k] and
 * expert_weights[top_k] (fp32) in device memory.  n_experts <= 4096,
 * top_k <= 32.  Experts sharded by id over shard_count GPUs: this GPU holds
 * experts e % shard_count == shard_index at local index e / shard_count; the
 * others get id -1 and weight 0 (skipped by the expert matvecs and the
 * combine).  global_ids (may be NULL) receives the global ids. */
int pyrite_cuda_moe_route(const float *router_logits, int n_experts, int top_k, int norm_topk_prob,
                          double scale, int shard_count, int shard_index, int *expert_ids,
                          float *expert_weights, int *global_ids, void *stream);

/* The router product (an F32 matrix of n_experts rows x hidden, type id 0, as
 * the reference stores it) and pyrite_cuda_moe_route in one launch:
 * router_logits receives the logits (accumulated in fp64 like the reference's
 * products, rounded to fp32 once), then the last CTA to finish routes.  `ticket`: one zeroed unsigned in
 * device memory, left at zero (one per concurrent call).  Other router types:
 * PYRITE_E_TYPE (use pyrite_cuda_matvec + pyrite_cuda_moe_route). */
int pyrite_cuda_moe_router_route(int router_type, const void *router, size_t router_len, size_t hidden,
                                 const float *x, float *router_logits, int n_experts, int top_k,
                                 int norm_topk_prob, double scale, int shard_count, int shard_index,
                                 int *expert_ids, float *expert_weights, int *global_ids, unsigned *ticket,
                                 void *stream);

/* As pyrite_cuda_moe_router_route with x the residual stream: the launch
 * also computes x' = RMSNorm(x) * norm_weight (fp64 statistics, as
 * pyrite_cuda_rmsnorm_encode), routes on W x', and writes x' to `normed` and
 * its encoding to `workspace` (as pyrite_cuda_rmsnorm_encode does) for the
 * expert products.  hidden % 32 == 0; router, x, norm_weight, normed 16-byte
 * aligned, workspace 256-byte aligned. */
int pyrite_cuda_moe_norm_router_route(int router_type, const void *router, size_t router_len, size_t hidden,
                                      const float *x, const float *norm_weight, double eps, float *normed,
                                      void *workspace, size_t workspace_len, float *router_logits,
                                      int n_experts, int top_k, int norm_topk_prob, double scale,
                                      int shard_count, int shard_index, int *expert_ids,
                                      float *expert_weights, int *global_ids, unsigned *ticket, void *stream);

/* The batch-1 product over n_sel routed slices of a stacked expert tensor in
 * one launch: `stacked` holds n_experts matrices of rows x cols back to back
 * (expert e at e * rows * row_bytes, qwen3_moe.py:364-398); expert_ids
 * (device, n_sel entries, written by an earlier kernel on the stream) pick the
 * slices; slice j multiplies the j-th activation -- x + j * x_stride in fp32
 * and its encoding at workspace + j * ws_stride (strides 0: one x for all, as
 * pyrite_cuda_prepare_x writes it) -- into y + j * y_stride.  Every decodable
 * type (the batch-1 kernel where it takes the format and alignment, else the
 * generic kernel on the fp32 x); id -1 skips the slice (an expert another GPU
 * holds); any other id outside [0, n_experts) reads expert 0 and sets status
 * bit 1. */
int pyrite_cuda_matvec_experts(int type_id, const void *stacked, size_t stacked_len, size_t n_experts,
                               const int *expert_ids, size_t n_sel, const float *x, size_t x_stride,
                               const void *workspace, size_t workspace_len, size_t ws_stride,
                               float *y, size_t y_stride, size_t rows, size_t cols, unsigned flags,
                               void *stream);

/* pyrite_cuda_matvec_experts over n_groups stacks of the same type and shape
 * stored back to back (e.g. ffn_gate_exps then ffn_up_exps: stacked_len =
 * n_groups * n_experts * rows * row_bytes), all in one launch: selection
 * j < n_groups * n_ids multiplies expert expert_ids[j % n_ids] of stack
 * j / n_ids by activation j % n_ids into y + j * y_stride.  n_groups <= 8,
 * n_groups * n_ids <= 1024. */
int pyrite_cuda_matvec_expert_groups(int type_id, const void *stacked, size_t stacked_len, size_t n_experts,
                                     size_t n_groups, const int *expert_ids, size_t n_ids, const float *x,
                                     size_t x_stride, const void *workspace, size_t workspace_len,
                                     size_t ws_stride, float *y, size_t y_stride, size_t rows, size_t cols,
                                     unsigned flags, void *stream);

/* pyrite_cuda_matvec_expert_groups for `count` sequences at once: expert_ids
 * holds each sequence's top_k experts (count x top_k, as
 * pyrite_cuda_moe_route_rows writes them), and selection j of a group
 * multiplies expert expert_ids[j] by the activation of sequence j / top_k --
 * x + (j / top_k) * x_stride and its encoding at workspace + (j / top_k) *
 * ws_stride (pyrite_cuda_prepare_x of the count rows) -- into y + (group *
 * count * top_k + j) * y_stride.  count * top_k * n_groups <= 1024. */
int pyrite_cuda_matvec_expert_rows(int type_id, const void *stacked, size_t stacked_len, size_t n_experts,
                                   size_t n_groups, const int *expert_ids, size_t count, size_t top_k,
                                   const float *x, size_t x_stride, const void *workspace, size_t workspace_len,
                                   size_t ws_stride, float *y, size_t y_stride, size_t rows, size_t cols,
                                   unsigned flags, void *stream);
/* The F32 router product (type id 0) of `count` sequences: router_logits[b *
 * ld + e] = W[e] . x[b * ldx ...], accumulated in fp64 and rounded to fp32
 * once, as pyrite_cuda_moe_router_route computes one sequence's. */
int pyrite_cuda_moe_router_rows(int router_type, const void *router, size_t router_len, size_t hidden,
                                const float *x, long long ldx, size_t count, float *router_logits, long long ld,
                                int n_experts, void *stream);
/* pyrite_cuda_moe_route for each row of a [count x n_experts] logits array (one
 * sequence per row): row j's experts and weights at expert_ids / expert_weights
 * + j * top_k (one GPU: no expert sharding). */
int pyrite_cuda_moe_route_rows(const float *router_logits, long long ld, size_t count, int n_experts, int top_k,
                               int norm_topk_prob, double scale, int *expert_ids, float *expert_weights,
                               void *stream);
/* Row b of hidden (ldh floats apart) += sum_j expert_weights[b top_k + j] *
 * expert_out[(b top_k + j) h ...], j ascending, for b < count. */
int pyrite_cuda_moe_combine_rows(const float *expert_out, const float *expert_weights, size_t top_k, size_t h,
                                 size_t count, float *hidden, long long ldh, void *stream);

/* act_j = silu(gate_j) * up_j for the n_sel experts (gate, up, act: n_sel x ff),
 * each encoded at workspace + j * pyrite_cuda_workspace_size(0, ff, 1). */
int pyrite_cuda_moe_silu_mul_encode(const float *gate, const float *up, size_t ff, size_t n_sel,
                                    float *act, void *workspace, size_t workspace_len, void *stream);

/* hidden[i] += sum_j expert_weights[j] * expert_out[j * h + i], j ascending. */
int pyrite_cuda_moe_combine(const float *expert_out, const float *expert_weights, size_t n_sel, size_t h,
                            float *hidden, void *stream);


/* ---- the decode step's sum across GPUs (tensor parallel) --------------------
 * The partial residual updates of the ranks (n floats each, after the output
 * and down projections) summed on every rank over NVLink peer memory, one
 * kernel per call; replaces the reference-free NCCL allreduce of the
 * sharded step (the reference runs on one host process).  Set-up, once per
 * rank: pyrite_cuda_ipc_buffer_create(pyrite_cuda_allreduce_buffer_size(n))
 * (zeroed), exchange the 64-byte handles, pyrite_cuda_ipc_buffer_open every
 * peer's, put the world device pointers (this rank's own at index rank) in a
 * device array `peer_buffers`, zero a device counter `epoch`, and let all
 * ranks pass a host barrier.  Every rank then makes the same calls in the
 * same order; inout += sum over ranks (rank order, identical bits on every
 * rank) of part.  n % 4 == 0, part and inout 16-byte aligned; buffer_len is
 * the size every rank's buffer was created with (n beyond what it holds is
 * PYRITE_E_BUFFER).  A wait longer than 5 s sets status bit 0 (see
 * pyrite_cuda_status) and returns. */
size_t pyrite_cuda_allreduce_buffer_size(size_t n);
int pyrite_cuda_ipc_buffer_create(size_t bytes, void **dev_ptr, void *handle_out);
int pyrite_cuda_ipc_buffer_open(const void *handle, void **dev_ptr);
int pyrite_cuda_ipc_buffer_close(void *dev_ptr, int owned);
int pyrite_cuda_allreduce_sum(const float *part, float *inout, size_t n,
                              const unsigned long long *peer_buffers, size_t buffer_len, int world,
                              int rank, unsigned *epoch, void *stream);

/* Static description of a return code. */
const char *pyrite_error_string(int code);

#ifdef __cplusplus
}
#endif

#endif /* PYRITE_B200_H */

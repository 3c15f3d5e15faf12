"""Locate, build on demand and bind libpyrite_b200.so (ctypes)."""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_native" / "libpyrite_b200.so"

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_attempted = False

_SZ = ctypes.c_size_t
_VP = ctypes.c_void_p
_PD = ctypes.POINTER(ctypes.c_double)

class PostOp(ctypes.Structure):
    """``pyrite_post_op`` (include/pyrite_b200.h)."""

    _fields_ = [("op", ctypes.c_int), ("prompt_len", ctypes.c_int), ("max_ctx", ctypes.c_int),
                ("eps", ctypes.c_double), ("weight", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_len", ctypes.c_size_t), ("ticket", ctypes.c_void_p),
                ("scratch", ctypes.c_void_p), ("scratch_len", ctypes.c_size_t), ("tokens", ctypes.c_void_p),
                ("pos", ctypes.c_void_p)]


POST_NONE, POST_RMSNORM_ENCODE, POST_SILU_MUL_ENCODE, POST_ARGMAX = 0, 1, 2, 3
X_RMSNORM, X_SILU_MUL = 1, 2  # pyrite_cuda_matvec_transformed

# name -> (restype, argtypes); exactly the symbols of include/pyrite_b200.h
SIGNATURES: dict[str, tuple] = {
    "pyrite_native_types": (ctypes.c_int, (ctypes.POINTER(ctypes.c_int), _SZ)),
    "pyrite_matvec": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _PD, _PD, _SZ, _SZ)),
    "pyrite_dequantize_rows": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _PD, _SZ, _SZ)),
    "pyrite_type_geometry": (ctypes.c_int, (ctypes.c_int, ctypes.POINTER(_SZ), ctypes.POINTER(_SZ))),
    "pyrite_cuda_workspace_size": (_SZ, (ctypes.c_int, _SZ, _SZ)),
    "pyrite_cuda_matvec": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, ctypes.c_longlong, _VP,
                                          ctypes.c_longlong, _SZ, _SZ, _SZ, ctypes.c_uint, _VP, _SZ, _VP)),
    "pyrite_cuda_prepare_x": (ctypes.c_int, (_VP, ctypes.c_longlong, _SZ, _SZ, _VP, _SZ, _VP)),
    "pyrite_cuda_matvec_prepared": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, _VP, _SZ, _VP, _SZ, _SZ,
                                                   ctypes.c_uint, _VP)),
    "pyrite_cuda_matvec_transformed": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, ctypes.c_int, _VP,
                                                      ctypes.c_double, _VP, _VP, _SZ, _VP, _SZ, _SZ, ctypes.c_uint,
                                                      _VP)),
    "pyrite_cuda_matvec_transformed_form": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, ctypes.c_int, _VP, _VP, _SZ,
                                                           _SZ)),
    "pyrite_cuda_post_scratch_size": (_SZ, ()),
    "pyrite_cuda_matvec_prepared_post": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, _VP, _SZ, _VP, _SZ, _SZ,
                                                        ctypes.c_uint, ctypes.POINTER(PostOp), _VP)),
    "pyrite_cuda_matvec_noalloc": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, _VP, _SZ, _SZ, ctypes.c_uint, _VP)),
    "pyrite_cuda_embed": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _VP, _VP, _VP, _VP)),
    "pyrite_cuda_rmsnorm_encode": (ctypes.c_int, (_VP, _VP, _SZ, ctypes.c_double, _VP, _VP, _SZ, _VP)),
    "pyrite_cuda_qk_rope_kv": (ctypes.c_int, (_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_double, _VP, _VP, ctypes.c_int, _VP, _VP, _VP, _VP)),
    "pyrite_cuda_attention": (ctypes.c_int, (_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, _VP, _VP)),
    "pyrite_cuda_attention_scratch_size": (_SZ, (ctypes.c_int, ctypes.c_int)),
    "pyrite_cuda_attention_step": (ctypes.c_int, (_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_double, _VP, _VP, ctypes.c_int, _VP, _VP, _VP, _VP, _SZ,
                                                  _VP, _SZ, _VP)),
    "pyrite_cuda_moe_route": (ctypes.c_int, (_VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                             ctypes.c_int, ctypes.c_int, _VP, _VP, _VP, _VP)),
    "pyrite_cuda_allreduce_buffer_size": (_SZ, (_SZ,)),
    "pyrite_cuda_ipc_buffer_create": (ctypes.c_int, (_SZ, _VP, _VP)),
    "pyrite_cuda_ipc_buffer_open": (ctypes.c_int, (_VP, _VP)),
    "pyrite_cuda_ipc_buffer_close": (ctypes.c_int, (_VP, ctypes.c_int)),
    "pyrite_cuda_embed_rows": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _VP, ctypes.c_longlong, _VP, _SZ, _VP, ctypes.c_longlong, _VP)),
    "pyrite_cuda_rmsnorm_rows": (ctypes.c_int, (_VP, ctypes.c_longlong, _VP, _SZ, _SZ, ctypes.c_double, _VP, ctypes.c_longlong, _VP)),
    "pyrite_cuda_qk_rope_kv_rows": (ctypes.c_int, (_VP, ctypes.c_longlong, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int, _VP, ctypes.c_int,
                                                   ctypes.c_longlong, ctypes.c_int, _VP, ctypes.c_int, _VP, ctypes.c_longlong, _VP, _VP, _VP)),
    "pyrite_cuda_attention_rows": (ctypes.c_int, (_VP, ctypes.c_longlong, _VP, _VP, ctypes.c_longlong, ctypes.c_int, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  _VP, ctypes.c_longlong, _VP)),
    "pyrite_cuda_argmax_rows": (ctypes.c_int, (_VP, ctypes.c_longlong, _SZ, _SZ, _VP, ctypes.c_longlong, _VP, ctypes.c_int, ctypes.c_int, _VP)),
    "pyrite_cuda_advance_pos": (ctypes.c_int, (_VP, _VP)),
    "pyrite_cuda_silu_mul_rows": (ctypes.c_int, (_VP, ctypes.c_longlong, _SZ, _SZ, _VP, ctypes.c_longlong, _VP)),
    "pyrite_cuda_argmax_local": (ctypes.c_int, (_VP, _SZ, ctypes.c_longlong, _VP, _SZ, _VP, _VP)),
    "pyrite_cuda_argmax_pick": (ctypes.c_int, (_VP, _SZ, _VP, _VP, ctypes.c_int, ctypes.c_int, _VP)),
    "pyrite_cuda_matvec_expert_rows": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _SZ, _VP, _SZ, _SZ, _VP, _SZ, _VP, _SZ,
                                                      _SZ, _VP, _SZ, _SZ, _SZ, ctypes.c_uint, _VP)),
    "pyrite_cuda_moe_router_rows": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _VP, ctypes.c_longlong, _SZ, _VP,
                                                   ctypes.c_longlong, ctypes.c_int, _VP)),
    "pyrite_cuda_moe_route_rows": (ctypes.c_int, (_VP, ctypes.c_longlong, _SZ, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, _VP, _VP,
                                                  _VP)),
    "pyrite_cuda_moe_combine_rows": (ctypes.c_int, (_VP, _VP, _SZ, _SZ, _SZ, _VP, ctypes.c_longlong, _VP)),
    "pyrite_cuda_allreduce_sum": (ctypes.c_int, (_VP, _VP, _SZ, _VP, _SZ, ctypes.c_int, ctypes.c_int, _VP, _VP)),
    "pyrite_cuda_moe_norm_router_route": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _VP, _VP, ctypes.c_double, _VP,
                                                         _VP, _SZ, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                         ctypes.c_double, ctypes.c_int, ctypes.c_int, _VP, _VP, _VP,
                                                         _VP, _VP)),
    "pyrite_cuda_moe_router_route": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _VP, _VP, ctypes.c_int, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_double, ctypes.c_int, ctypes.c_int, _VP,
                                                    _VP, _VP, _VP, _VP)),
    "pyrite_cuda_matvec_experts": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _VP, _SZ, _VP, _SZ, _VP, _SZ, _SZ,
                                                  _VP, _SZ, _SZ, _SZ, ctypes.c_uint, _VP)),
    "pyrite_cuda_matvec_expert_groups": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _SZ, _SZ, _VP, _SZ, _VP, _SZ, _VP,
                                                        _SZ, _SZ, _VP, _SZ, _SZ, _SZ, ctypes.c_uint, _VP)),
    "pyrite_cuda_moe_silu_mul_encode": (ctypes.c_int, (_VP, _VP, _SZ, _SZ, _VP, _VP, _SZ, _VP)),
    "pyrite_cuda_moe_combine": (ctypes.c_int, (_VP, _VP, _SZ, _SZ, _VP, _VP)),
    "pyrite_cuda_silu_mul_encode": (ctypes.c_int, (_VP, _SZ, _VP, _VP, _SZ, _VP)),
    "pyrite_cuda_argmax_step": (ctypes.c_int, (_VP, _SZ, _VP, _SZ, _VP, _VP, ctypes.c_int, ctypes.c_int, _VP)),
    "pyrite_cuda_dequantize_rows": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, _SZ, _SZ, _VP)),
    "pyrite_cuda_device_count": (ctypes.c_int, ()),
    "pyrite_cuda_status": (ctypes.c_int, (ctypes.c_int,)),
    "pyrite_error_string": (ctypes.c_char_p, (ctypes.c_int,)),
    "pyrite_quantize": (ctypes.c_int, (ctypes.c_int, _VP, _SZ, _VP, _SZ, ctypes.c_int)),
    "pyrite_quantize_types": (ctypes.c_int, (ctypes.POINTER(ctypes.c_int), _SZ)),
}


def bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def load(build_if_missing: bool = True) -> ctypes.CDLL | None:
    """The bound library, or None when it is absent and cannot be built."""
    global _lib, _attempted
    with _lock:
        if _lib is not None or _attempted:
            return _lib
        _attempted = True
        if not LIB_PATH.is_file() and build_if_missing:
            try:
                from .build import build
                build()
            except Exception:  # noqa: BLE001 - no toolkit: report "unavailable"
                return None
        if not LIB_PATH.is_file():
            return None
        _lib = bind(ctypes.CDLL(str(LIB_PATH)))
        return _lib


def require() -> ctypes.CDLL:
    lib = load()
    if lib is None:
        raise RuntimeError(f"libpyrite_b200.so is not built ({LIB_PATH}); run python -m pyrite_b200.build")
    return lib


def type_ids(lib: ctypes.CDLL) -> list[int]:
    n = lib.pyrite_native_types(None, 0)
    buf = (ctypes.c_int * max(n, 0))()
    got = lib.pyrite_native_types(buf, n)
    return [buf[i] for i in range(max(0, got))]


def device_count() -> int:
    lib = load()
    return 0 if lib is None else int(lib.pyrite_cuda_device_count())


def error_string(code: int) -> str:
    lib = load()
    return lib.pyrite_error_string(code).decode() if lib is not None else f"error {code}"

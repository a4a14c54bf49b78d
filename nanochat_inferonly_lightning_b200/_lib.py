"""Loads libnanochat_attn_sm100.so and declares the C ABI of include/nanochat_attn.h.

There is no fallback: if the library is missing or fails to load, every entry point raises.
"""
import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libnanochat_attn_sm100.so")

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t
c_longlong = ctypes.c_longlong

# name -> (restype, argtypes); mirrors include/nanochat_attn.h one to one.
SIGNATURES = {
    "nc_status_string": (ctypes.c_char_p, [c_int]),
    "nc_last_cuda_error": (c_int, []),
    "nc_last_status": (c_int, []),
    "nc_device_status": (c_int, [c_int]),
    "nc_init_rope_tables": (c_int, []),
    "nc_apply_rope": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p]),
    "nc_apply_rope_rmsnorm": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p]),
    "nc_rope_qknorm_append": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int, c_int, c_int, c_void_p]),
    "nc_flash_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                   c_int, c_float, c_int, c_void_p]),
    "nc_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "nc_decode_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_int, c_int, c_float, c_int, c_int,
                                    c_void_p, c_size_t, c_void_p]),
    "nc_decode_attention_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_int, c_int, c_void_p, c_int, c_void_p,
                                          c_int, c_int, c_float, c_int, c_int, c_void_p,
                                          c_size_t, c_void_p]),
    "nc_decode_attention_overlap": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_void_p, c_int, c_int, c_float, c_int,
                                            c_int, c_void_p, c_size_t, c_void_p]),
    "nc_decode_attention_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_void_p, c_void_p, c_int, c_int, c_float, c_int,
                                            c_void_p]),
    "nc_rope_qknorm_append_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p,
                                              c_void_p, c_longlong, c_int, c_int, c_int, c_int,
                                              c_void_p]),
    "nc_rope_qknorm_append_paged_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p,
                                                    c_void_p, c_int, c_int, c_void_p, c_int,
                                                    c_int, c_int, c_int, c_int, c_void_p]),
    "nc_prefill_attention_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p,
                                             c_longlong, c_int, c_void_p, c_int, c_int, c_int,
                                             c_float, c_void_p]),
    "nc_rope_qknorm_append_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                            c_int, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                            c_void_p]),
    "nc_prefill_attention_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                           c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                           c_float, c_void_p]),
    "nc_kv_cache_create": (c_int, [ctypes.POINTER(c_void_p), c_int, c_int, c_int, c_int]),
    "nc_kv_cache_destroy": (c_int, [c_void_p]),
    "nc_kv_cache_k": (c_void_p, [c_void_p, c_int, c_int]),
    "nc_kv_cache_v": (c_void_p, [c_void_p, c_int, c_int]),
    "nc_kv_cache_k_table": (c_void_p, [c_void_p, c_int]),
    "nc_kv_cache_v_table": (c_void_p, [c_void_p, c_int]),
    "nc_kv_cache_seq_stride": (c_longlong, [c_void_p]),
    "nc_kv_cache_max_len": (c_int, [c_void_p]),
    "nc_kv_cache_len": (c_int, [c_void_p, c_int, c_int]),
    "nc_kv_cache_set_len": (c_int, [c_void_p, c_int, c_int, c_int]),
    "nc_kv_cache_clear": (c_int, [c_void_p, c_int]),
    "nc_kv_cache_prefill": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_int, c_float, c_void_p]),
    "nc_kv_cache_decode": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_float, c_void_p]),
    "nc_embed_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "nc_argmax_rows": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "nc_sample_rows": (c_int, [c_void_p, c_void_p, c_int, c_int, c_float, c_int, c_float,
                               c_void_p, c_void_p]),
    "nc_gemm_skinny": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                               c_int, c_float, c_int, c_int, c_void_p]),
    "nc_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                        c_float, c_int, c_void_p]),
}

# C++ entry points with the reference's names (namespace nanochat, C++ linkage).
DROPIN_SYMBOLS = {
    "apply_rope": "_ZN8nanochat10apply_ropeEP13__nv_bfloat16iiiP11CUstream_st",
    "apply_rope_rmsnorm": "_ZN8nanochat18apply_rope_rmsnormEP13__nv_bfloat16iiiP11CUstream_st",
    "init_rope_tables": "_ZN8nanochat16init_rope_tablesEv",
    "flash_attention": "_ZN8nanochat15flash_attentionEP13__nv_bfloat16PKS0_S3_S3_iiifiP11CUstream_st",
}

_lib = None


class NcError(RuntimeError):
    """A library call returned a non-zero nc_status."""

    def __init__(self, fn, status, lib=None):
        text = lib.nc_status_string(status).decode() if lib is not None else str(status)
        extra = ""
        if lib is not None and status == 3:
            extra = f" (cudaError {lib.nc_last_cuda_error()})"
        super().__init__(f"{fn} failed: {text}{extra}")
        self.status = status


def load(path=None):
    """Returns the loaded library (loading it on first use).  Raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(
            f"{p} is missing: build it with `python -m nanochat_inferonly_lightning_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(fn_name, status):
    if status != 0:
        raise NcError(fn_name, status, _lib)

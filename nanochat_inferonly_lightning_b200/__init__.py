"""B200-native (sm_100a) attention hot path of the nanochat inference engine, and the skinny
tcgen05 GEMM of its decode step (gemm.py).

The compute lives in libnanochat_attn_sm100.so (CUDA kernels + C ABI, include/nanochat_attn.h);
this package is the Python-side mirror of the reference's entry points over that ABI.
Importing it does not load the library; the first call does, and raises if it is missing.
"""
from ._lib import LIB_PATH, NcError, load
from . import gemm
from .attn import (HEAD_DIM, ROPE_MAX_SEQ, KVCache, apply_rope, apply_rope_rmsnorm,
                   decode_attention, decode_attention_paged, decode_workspace_bytes, device_status, flash_attention,
                   init_rope_tables, prefill_attention_batched, prefill_attention_paged,
                   rope_qknorm_append, rope_qknorm_append_batched, rope_qknorm_append_paged,
                   rope_qknorm_append_paged_batched)

__all__ = [
    "LIB_PATH", "NcError", "load", "HEAD_DIM", "ROPE_MAX_SEQ", "KVCache", "apply_rope",
    "apply_rope_rmsnorm", "decode_attention", "decode_attention_paged", "decode_workspace_bytes", "device_status",
    "flash_attention", "init_rope_tables", "prefill_attention_batched", "prefill_attention_paged", "rope_qknorm_append",
    "rope_qknorm_append_batched", "rope_qknorm_append_paged", "rope_qknorm_append_paged_batched",
    "gemm",
]

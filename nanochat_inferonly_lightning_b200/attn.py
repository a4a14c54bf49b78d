"""Python mirror of the reference engine's attention entry points, over the C ABI.

Names, argument order and meaning follow the reference's declarations in src/model.h:14-16,
26-27 (apply_rope, apply_rope_rmsnorm, init_rope_tables, flash_attention); tensors are torch
CUDA bf16 tensors laid out as in the reference ([rows, heads, 128], out [rows, heads*128]).
The reference's functions return nothing and never report errors; these raise NcError on a
non-zero status instead.  The stream defaults to torch's current stream.
"""
import ctypes

import torch

from . import _lib

HEAD_DIM = 128
ROPE_MAX_SEQ = 20480


def _stream(stream):
    if stream is None:
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, torch.cuda.Stream):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


def _ptr(t):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor):
        return ctypes.c_void_p(int(t))
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return ctypes.c_void_p(t.data_ptr())


def _bf16(*ts):
    for t in ts:
        if t is not None and isinstance(t, torch.Tensor) and t.dtype != torch.bfloat16:
            raise TypeError(f"expected bfloat16, got {t.dtype}")


def init_rope_tables():
    """kernels/rope.cu:14-30: builds and uploads the cos/sin table for the current device."""
    lib = _lib.load()
    _lib.check("nc_init_rope_tables", lib.nc_init_rope_tables())


def apply_rope(x, seq_len, n_heads, start_pos, stream=None):
    """kernels/rope.cu:34-68: in-place half-split RoPE of x [seq_len, n_heads, 128]."""
    _bf16(x)
    lib = _lib.load()
    _lib.check("nc_apply_rope",
               lib.nc_apply_rope(_ptr(x), seq_len, n_heads, start_pos, _stream(stream)))


def apply_rope_rmsnorm(x, seq_len, n_heads, start_pos, stream=None):
    """kernels/rope.cu:74-158: in-place RoPE + parameter-free per-head RMSNorm (eps 1e-6)."""
    _bf16(x)
    lib = _lib.load()
    _lib.check("nc_apply_rope_rmsnorm",
               lib.nc_apply_rope_rmsnorm(_ptr(x), seq_len, n_heads, start_pos, _stream(stream)))


def rope_qknorm_append(q, k, v, k_cache, v_cache, seq_len, heads, start_pos, stream=None):
    """src/model.cpp:119-131 in one pass: q <- RoPE+QK-norm(q) in place; RoPE+QK-norm(k) and v
    land in cache rows [start_pos, start_pos + seq_len)."""
    _bf16(q, k, v, k_cache, v_cache)
    lib = _lib.load()
    _lib.check("nc_rope_qknorm_append",
               lib.nc_rope_qknorm_append(_ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache),
                                         seq_len, heads, start_pos, _stream(stream)))


def rope_qknorm_append_batched(q, k, v, k_slab, v_slab, seq_stride, batch, seq_len, heads,
                               start_pos, stream=None):
    """nc_rope_qknorm_append_batched: rope_qknorm_append for `batch` sequences in one launch.
    q, k, v are [batch * seq_len, heads, 128]; sequence b's cache starts seq_stride elements
    after sequence b-1's in k_slab / v_slab."""
    _bf16(q, k, v, k_slab, v_slab)
    lib = _lib.load()
    _lib.check("nc_rope_qknorm_append_batched",
               lib.nc_rope_qknorm_append_batched(_ptr(q), _ptr(k), _ptr(v), _ptr(k_slab),
                                                 _ptr(v_slab), int(seq_stride), batch, seq_len,
                                                 heads, start_pos, _stream(stream)))


def flash_attention(out, Q, K, V, seq_q, kv_len, heads, scale, kv_offset, stream=None):
    """kernels/flash_attention.cu:159-171: causal attention of Q [seq_q, heads, 128] over the
    cache K/V [>= kv_len, heads, 128]; key j is visible to query s iff j < kv_len and
    j <= s + kv_offset.  out [seq_q, heads*128]."""
    _bf16(out, Q, K, V)
    lib = _lib.load()
    _lib.check("nc_flash_attention",
               lib.nc_flash_attention(_ptr(out), _ptr(Q), _ptr(K), _ptr(V), seq_q, kv_len, heads,
                                      float(scale), kv_offset, _stream(stream)))


def decode_workspace_bytes(batch, max_kv_len, heads, split_len=0):
    return int(_lib.load().nc_decode_workspace_bytes(batch, max_kv_len, heads, split_len))


def decode_attention(out, q, k_new, v_new, k_ptrs, v_ptrs, kv_len, heads, scale, max_kv_len,
                     workspace, split_len=0, stream=None, overlap=False):
    """Batched decode step (include/nanochat_attn.h nc_decode_attention).

    k_ptrs/v_ptrs: int64 CUDA tensors [B] of per-sequence cache base addresses; kv_len: int32
    CUDA tensor [B]; workspace: a zero-filled uint8 CUDA tensor of at least
    decode_workspace_bytes(B, max_kv_len, heads, split_len) bytes.  overlap=True calls
    nc_decode_attention_overlap: only right after a kernel that writes none of the caches,
    kv_len or the pointer arrays (e.g. the Q/K/V projection)."""
    _bf16(out, q, k_new, v_new)
    batch = int(kv_len.numel())
    lib = _lib.load()
    name = "nc_decode_attention_overlap" if overlap else "nc_decode_attention"
    _lib.check(name,
               getattr(lib, name)(_ptr(out), _ptr(q), _ptr(k_new), _ptr(v_new), _ptr(k_ptrs),
                                  _ptr(v_ptrs), _ptr(kv_len), batch, heads, float(scale),
                                  max_kv_len, split_len, _ptr(workspace),
                                  workspace.numel() if workspace is not None else 0,
                                  _stream(stream)))


def decode_attention_paged(out, q, k_new, v_new, k_pool, v_pool, page_table, kv_len, heads,
                           scale, max_kv_len, workspace, split_len=0, stream=None):
    """Batched decode step over a paged cache (nc_decode_attention_paged).

    k_pool/v_pool: bf16 CUDA tensors [num_pages, page_rows, heads, 128]; page_table: int32 CUDA
    tensor [B, pages_per_seq] of page ids; kv_len: int32 CUDA tensor [B]."""
    _bf16(out, q, k_new, v_new, k_pool, v_pool)
    if page_table.dtype != torch.int32 or page_table.dim() != 2:
        raise TypeError("page_table must be an int32 tensor [batch, pages_per_seq]")
    batch = int(kv_len.numel())
    num_pages, page_rows = int(k_pool.shape[0]), int(k_pool.shape[1])
    lib = _lib.load()
    _lib.check("nc_decode_attention_paged",
               lib.nc_decode_attention_paged(_ptr(out), _ptr(q), _ptr(k_new), _ptr(v_new),
                                             _ptr(k_pool), _ptr(v_pool), num_pages, page_rows,
                                             _ptr(page_table), int(page_table.shape[1]),
                                             _ptr(kv_len), batch, heads, float(scale),
                                             max_kv_len, split_len, _ptr(workspace),
                                             workspace.numel() if workspace is not None else 0,
                                             _stream(stream)))


def rope_qknorm_append_paged(q, k, v, k_pool, v_pool, pages, seq_len, heads, start_pos,
                             stream=None):
    """nc_rope_qknorm_append_paged: q gets RoPE + QK-norm in place; k (after RoPE + QK-norm) and
    v land at positions start_pos.. of the sequence whose pages are `pages` (host list of page
    ids, in position order) in the pools [num_pages, page_rows, heads, 128]."""
    _bf16(q, k, v, k_pool, v_pool)
    ids = (ctypes.c_int * len(pages))(*[int(x) for x in pages])
    lib = _lib.load()
    _lib.check("nc_rope_qknorm_append_paged",
               lib.nc_rope_qknorm_append_paged(_ptr(q), _ptr(k), _ptr(v), _ptr(k_pool),
                                               _ptr(v_pool), int(k_pool.shape[0]),
                                               int(k_pool.shape[1]), ids, len(pages), seq_len,
                                               heads, start_pos, _stream(stream)))


def rope_qknorm_append_paged_batched(q, k, v, k_pool, v_pool, page_table, seq_len, heads,
                                     start_pos, stream=None):
    """nc_rope_qknorm_append_paged_batched: rope_qknorm_append_paged for every row of the device
    page table (int32 CUDA [B, pages_per_seq]) in one launch; q, k, v are [B * seq_len, heads,
    128]."""
    _bf16(q, k, v, k_pool, v_pool)
    if page_table.dtype != torch.int32 or not page_table.is_cuda or not page_table.is_contiguous():
        raise ValueError("page_table must be a contiguous int32 CUDA tensor")
    lib = _lib.load()
    _lib.check("nc_rope_qknorm_append_paged_batched",
               lib.nc_rope_qknorm_append_paged_batched(
                   _ptr(q), _ptr(k), _ptr(v), _ptr(k_pool), _ptr(v_pool), int(k_pool.shape[0]),
                   int(k_pool.shape[1]), _ptr(page_table), int(page_table.shape[1]),
                   int(page_table.shape[0]), seq_len, heads, start_pos, _stream(stream)))


def prefill_attention_paged(out, q, k_pool, v_pool, page_table, kv_offset, seq_q, heads, scale,
                            stream=None):
    """nc_prefill_attention_paged: causal chunked prefill of q [B, seq_q, heads, 128] over keys
    read through page_table (int32 CUDA [B, pages_per_seq]); kv_offset int32 CUDA [B]."""
    _bf16(out, q, k_pool, v_pool)
    batch = int(kv_offset.numel())
    lib = _lib.load()
    _lib.check("nc_prefill_attention_paged",
               lib.nc_prefill_attention_paged(_ptr(out), _ptr(q), _ptr(k_pool), _ptr(v_pool),
                                              int(k_pool.shape[0]), int(k_pool.shape[1]),
                                              _ptr(page_table), int(page_table.shape[1]),
                                              _ptr(kv_offset), batch, seq_q, heads, float(scale),
                                              _stream(stream)))


def prefill_attention_batched(out, q, k_slab, v_slab, seq_stride, rows_per_seq, kv_offset,
                              seq_q, heads, scale, stream=None):
    """Batched chunked prefill over caches that are slices of one slab (seq_stride elements
    apart); kv_offset: int32 CUDA tensor [B]."""
    _bf16(out, q, k_slab, v_slab)
    batch = int(kv_offset.numel())
    lib = _lib.load()
    _lib.check("nc_prefill_attention_batched",
               lib.nc_prefill_attention_batched(_ptr(out), _ptr(q), _ptr(k_slab), _ptr(v_slab),
                                                int(seq_stride), rows_per_seq, _ptr(kv_offset),
                                                batch, seq_q, heads, float(scale),
                                                _stream(stream)))


def device_status(reset=False):
    """Kernel status word of the current device (non-zero: a bounded wait gave up)."""
    return int(_lib.load().nc_device_status(1 if reset else 0))


class KVCache:
    """Per-layer KV slabs [n_seqs, max_len, heads, 128] bf16, allocated once at full length
    (replaces KVCache, src/model.h:65-73, and its grow-and-copy, src/model.cpp:52-81)."""

    def __init__(self, n_layers, n_seqs, max_len, heads):
        lib = _lib.load()
        h = ctypes.c_void_p()
        _lib.check("nc_kv_cache_create",
                   lib.nc_kv_cache_create(ctypes.byref(h), n_layers, n_seqs, max_len, heads))
        self._h = h
        self.n_layers, self.n_seqs, self.max_len, self.heads = n_layers, n_seqs, max_len, heads

    def close(self):
        if self._h:
            _lib.check("nc_kv_cache_destroy", _lib.load().nc_kv_cache_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def k_ptr(self, layer, seq):
        return _lib.load().nc_kv_cache_k(self._h, layer, seq)

    def v_ptr(self, layer, seq):
        return _lib.load().nc_kv_cache_v(self._h, layer, seq)

    @property
    def seq_stride(self):
        return int(_lib.load().nc_kv_cache_seq_stride(self._h))

    def length(self, layer, seq):
        return int(_lib.load().nc_kv_cache_len(self._h, layer, seq))

    def set_length(self, layer, seq, n):
        _lib.check("nc_kv_cache_set_len", _lib.load().nc_kv_cache_set_len(self._h, layer, seq, n))

    def clear(self, seq=-1):
        _lib.check("nc_kv_cache_clear", _lib.load().nc_kv_cache_clear(self._h, seq))

    def view(self, layer, seq, which="k"):
        """A torch view of one sequence's rows [max_len, heads, 128] (shares memory)."""
        ptr = self.k_ptr(layer, seq) if which == "k" else self.v_ptr(layer, seq)
        return _wrap_device(ptr, (self.max_len, self.heads, HEAD_DIM))

    def prefill(self, layer, seq, out, q, k, v, seq_len, scale, stream=None):
        _bf16(out, q, k, v)
        _lib.check("nc_kv_cache_prefill",
                   _lib.load().nc_kv_cache_prefill(self._h, layer, seq, _ptr(out), _ptr(q), _ptr(k),
                                                   _ptr(v), seq_len, float(scale), _stream(stream)))

    def decode(self, layer, out, q, k_new, v_new, scale, stream=None):
        _bf16(out, q, k_new, v_new)
        _lib.check("nc_kv_cache_decode",
                   _lib.load().nc_kv_cache_decode(self._h, layer, _ptr(out), _ptr(q), _ptr(k_new),
                                                  _ptr(v_new), float(scale), _stream(stream)))


def _wrap_device(ptr, shape):
    """Wraps library-owned device memory as a bf16 torch tensor (no copy, no ownership)."""

    class _Holder:
        pass

    holder = _Holder()
    n = 1
    for d in shape:
        n *= d
    holder.__cuda_array_interface__ = {
        "shape": (n,), "typestr": "<u2", "data": (int(ptr), False), "version": 3,
    }
    t = torch.as_tensor(holder, device="cuda").view(torch.bfloat16)
    return t.view(*shape)

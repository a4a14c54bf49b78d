"""TEST INFRASTRUCTURE ONLY: ctypes access to the C oracle (nc_oracle.c) and to the
reference's own kernels rebuilt for sm_100a (oracle/_ref/libref_attn.so).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs use this.
bf16 tensors are numpy uint16 arrays of bit patterns.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libnc_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_attn.so")
HEAD_DIM = 128
ROPE_MAX_SEQ = 20480

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_orc = None
_ref = None


def _ptr(a):
    return a.ctypes.data_as(_P)


def oracle():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            from . import build as _b
            _b.build(verbose=False)
        lib = ctypes.CDLL(ORACLE_SO)
        lib.orc_rope_tables.argtypes = [_P, _P, _I]
        lib.orc_apply_rope.argtypes = [_P, _I, _I, _I, _P, _P]
        lib.orc_apply_rope_rmsnorm.argtypes = [_P, _I, _I, _I, _P, _P]
        lib.orc_rope_qknorm_append.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P]
        lib.orc_flash_attention.argtypes = [_P, _P, _P, _P, _I, _I, _I, _F, _I]
        lib.orc_decode_step.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I, _I, _F, _P, _P]
        lib.orc_sample.argtypes = [_P, _I, _F, _I, _F, _F]
        lib.orc_sample.restype = _I
        for f in ("orc_rope_tables", "orc_apply_rope", "orc_apply_rope_rmsnorm",
                  "orc_rope_qknorm_append", "orc_flash_attention", "orc_decode_step"):
            getattr(lib, f).restype = None
        _orc = lib
    return _orc


_tables = {}


def rope_tables(max_pos=ROPE_MAX_SEQ):
    """(cos, sin) fp32 [max_pos, 64] as the reference builds them (kernels/rope.cu:14-30)."""
    if max_pos not in _tables:
        c = np.zeros((max_pos, 64), np.float32)
        s = np.zeros((max_pos, 64), np.float32)
        oracle().orc_rope_tables(_ptr(c), _ptr(s), max_pos)
        _tables[max_pos] = (c, s)
    return _tables[max_pos]


def _u16(a):
    a = np.ascontiguousarray(a)
    assert a.dtype == np.uint16
    return a


def apply_rope(x, seq_len, heads, start_pos):
    x = _u16(x).copy()
    c, s = rope_tables()
    oracle().orc_apply_rope(_ptr(x), seq_len, heads, start_pos, _ptr(c), _ptr(s))
    return x


def apply_rope_rmsnorm(x, seq_len, heads, start_pos):
    x = _u16(x).copy()
    c, s = rope_tables()
    oracle().orc_apply_rope_rmsnorm(_ptr(x), seq_len, heads, start_pos, _ptr(c), _ptr(s))
    return x


def rope_qknorm_append(q, k, v, k_cache, v_cache, seq_len, heads, start_pos):
    """Returns (q', k_cache', v_cache') without modifying the inputs."""
    q = _u16(q).copy()
    kc = _u16(k_cache).copy()
    vc = _u16(v_cache).copy()
    c, s = rope_tables()
    oracle().orc_rope_qknorm_append(_ptr(q), _ptr(_u16(k)), _ptr(_u16(v)), _ptr(kc), _ptr(vc),
                                    seq_len, heads, start_pos, _ptr(c), _ptr(s))
    return q, kc, vc


def flash_attention(Q, K, V, seq_q, kv_len, heads, scale, kv_offset):
    out = np.zeros((seq_q, heads * HEAD_DIM), np.uint16)
    oracle().orc_flash_attention(_ptr(out), _ptr(_u16(Q)), _ptr(_u16(K)), _ptr(_u16(V)), seq_q,
                                 kv_len, heads, float(scale), kv_offset)
    return out


def decode_step(q, k_new, v_new, k_caches, v_caches, kv_len, heads, scale):
    """Fused decode step over a list of per-sequence caches; returns (out, k_caches',
    v_caches') without modifying the inputs."""
    batch = len(kv_len)
    kcs = [_u16(k).copy() for k in k_caches]
    vcs = [_u16(v).copy() for v in v_caches]
    kp = (_P * batch)(*[k.ctypes.data for k in kcs])
    vp = (_P * batch)(*[v.ctypes.data for v in vcs])
    lens = np.ascontiguousarray(np.asarray(kv_len, np.int32))
    out = np.zeros((batch, heads * HEAD_DIM), np.uint16)
    c, s = rope_tables()
    oracle().orc_decode_step(_ptr(out), _ptr(_u16(q)),
                             _ptr(_u16(k_new)) if k_new is not None else None,
                             _ptr(_u16(v_new)) if v_new is not None else None,
                             ctypes.cast(kp, _P), ctypes.cast(vp, _P), _ptr(lens), batch, heads,
                             float(scale), _ptr(c), _ptr(s))
    return out, kcs, vcs


def sample(logits_row, temperature, top_k, top_p, r):
    """Engine::sample (src/engine.cpp:88-131) of one bf16 logits row (uint16 bits) with the
    uniform draw r given; equal probabilities ordered by index."""
    row = _u16(logits_row)
    return int(oracle().orc_sample(_ptr(row), row.size, float(temperature), int(top_k),
                                   float(top_p), float(r)))


def reference_kernels():
    """The reference's own CUDA kernels (rebuilt for sm_100a), or None if not built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            return None
        lib = ctypes.CDLL(REF_SO)
        lib.ref_init_rope_tables.argtypes = []
        lib.ref_get_rope_tables.argtypes = [_P, _P, _I]
        lib.ref_apply_rope.argtypes = [_P, _I, _I, _I, _P]
        lib.ref_apply_rope_rmsnorm.argtypes = [_P, _I, _I, _I, _P]
        lib.ref_flash_attention.argtypes = [_P, _P, _P, _P, _I, _I, _I, _F, _I, _P]
        lib.ref_rmsnorm.argtypes = [_P, _P, _I, _I, _P]
        lib.ref_embedding.argtypes = [_P, _P, _P, _I, _I, _P]
        lib.ref_relu_squared.argtypes = [_P, _I, _P]
        lib.ref_tanh_cap.argtypes = [_P, _I, _F, _P]
        for f in ("ref_init_rope_tables", "ref_get_rope_tables", "ref_apply_rope",
                  "ref_apply_rope_rmsnorm", "ref_flash_attention", "ref_rmsnorm",
                  "ref_embedding", "ref_relu_squared", "ref_tanh_cap"):
            getattr(lib, f).restype = _I
        _ref = lib
    return _ref


def bf16_bits_to_f32(a):
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a):
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(np.asarray(a, np.float32)).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r

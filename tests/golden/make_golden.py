"""Generates tests/golden/reference_kernels.npz: inputs and outputs of the reference's own CUDA
kernels (kernels/rope.cu, kernels/flash_attention.cu of the reference project, rebuilt for
sm_100a into oracle/_ref/libref_attn.so by oracle/build_ref.py), run on a B200.

These are the golden vectors the CPU oracle is pinned against (tests/test_oracle_cpu.py).
Run on a GPU box from the repository root:
    python tests/golden/make_golden.py [output.npz]
Inputs are seeded normal draws (numpy default_rng); Q/K for attention are normalised by the
reference's own apply_rope_rmsnorm first, as the engine does (src/model.cpp:119-120).
"""
import ctypes
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
import oracle  # noqa: E402

H, D = 17, 128
SCALE = np.float32(1.0 / np.sqrt(128.0))
OUT = os.path.join(ROOT, "tests", "golden", "reference_kernels.npz")


def rand_u16(shape, seed):
    rng = np.random.default_rng(seed)
    return oracle.f32_to_bf16_bits(rng.standard_normal(shape).astype(np.float32))


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def to_host(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16).copy()


def main(path=OUT):
    ref = oracle.reference_kernels()
    assert ref is not None, "build oracle/_ref first (python oracle/build_ref.py)"
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    assert ref.ref_init_rope_tables() == 0
    res = {}

    pos = np.array([0, 1, 2, 3, 255, 511, 512, 1023, 1024, 2047, 2048, 4095, 8191, 10000,
                    16384, 20479], np.int64)
    c = np.zeros((20480, 64), np.float32)
    sn = np.zeros((20480, 64), np.float32)
    assert ref.ref_get_rope_tables(c.ctypes.data_as(ctypes.c_void_p),
                                   sn.ctypes.data_as(ctypes.c_void_p), 20480) == 0
    res["table_positions"] = pos
    res["table_cos"] = c[pos]
    res["table_sin"] = sn[pos]

    for name, seq_len, start, fn in (("rope", 16, 1000, ref.ref_apply_rope),
                                     ("rope_rmsnorm", 16, 511, ref.ref_apply_rope_rmsnorm)):
        x = rand_u16((seq_len, H, D), 100 + seq_len + start)
        t = to_dev(x)
        assert fn(P(t), seq_len, H, start, s) == 0
        torch.cuda.synchronize()
        res[f"{name}_in"] = x
        res[f"{name}_out"] = to_host(t)
        res[f"{name}_args"] = np.array([seq_len, start], np.int64)

    cases = {
        "attn_decode": (1, 130, 129),
        "attn_decode_limited": (1, 64, 20),
        "attn_prefill_small": (8, 8, 0),
        "attn_prefill_33": (33, 33, 0),
        "attn_chunk_offset": (40, 72, 32),
        "attn_no_visible": (3, 5, -1),
    }
    for i, (n, (seq_q, kv_len, off)) in enumerate(cases.items()):
        q = rand_u16((seq_q, H, D), 200 + i)
        k = rand_u16((kv_len, H, D), 300 + i)
        v = rand_u16((kv_len, H, D), 400 + i)
        tq, tk, tv = to_dev(q), to_dev(k), to_dev(v)
        assert ref.ref_apply_rope_rmsnorm(P(tq), seq_q, H, max(off, 0), s) == 0
        assert ref.ref_apply_rope_rmsnorm(P(tk), kv_len, H, 0, s) == 0
        out = torch.empty((seq_q, H * D), dtype=torch.bfloat16, device="cuda")
        assert ref.ref_flash_attention(P(out), P(tq), P(tk), P(tv), seq_q, kv_len, H,
                                       float(SCALE), off, s) == 0
        torch.cuda.synchronize()
        res[n + "_q"] = to_host(tq)
        res[n + "_k"] = to_host(tk)
        res[n + "_v"] = v
        res[n + "_out"] = to_host(out)
        res[n + "_args"] = np.array([seq_q, kv_len, off], np.int64)
    np.savez_compressed(path, **res)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else OUT)

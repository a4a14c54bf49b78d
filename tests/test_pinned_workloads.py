"""Parity on the exact inputs and launches whose throughput bench.py reports.

Each case draws its inputs from the same workloads.py generators and seeds as bench.py's first
input set on rank 0, prepares them the way the bench does (cache keys RoPE + QK-normalised by
this library's kernel), makes the same C-ABI calls with the same arguments, and compares the
result with the CPU oracle (oracle/nc_oracle.c) at the north-star tolerance (max-abs 2e-2,
mean-abs 2e-3 on bf16 outputs).  Appended cache rows and normalised queries are checked too
(RoPE + QK-norm within one bf16 ulp of the oracle; values copied exactly).

  cfg1  decode, 1 sequence, query at position 511 (cfg1_inputs, seed 0)
  cfg2  prefill, 2048 positions (cfg2_inputs, seed 1): RoPE/QK-norm/append pass + attention
  cfg3  decode, all 64 sequences of the seed-2 length draw, one launch, automatic splits
  cfg4  chunked prefill, 4 sequences x 512 queries at offset 1536 (seed 3 chunk, seed 30 cache)
"""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import assert_close_bf16, bf16_to_u16, ulp_diff_bf16

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from nanochat_inferonly_lightning_b200 import workloads as W  # noqa: E402

H, D, ROW = W.HEADS, W.HEAD_DIM, W.ROW


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc

    nc.init_rope_tables()
    yield nc.load()
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) == 0, "a kernel's bounded wait gave up"


def _normalise(lib, x, start_pos=0):
    """RoPE + QK-norm in place with this library's kernel (the bench's input preparation)."""
    assert lib.nc_apply_rope_rmsnorm(_p(x), x.shape[0], H, start_pos, _s()) == 0


def _decode_and_check(lib, q, kn, vn, kcs, vcs, lens, what):
    """bench.py's decode launch (automatic splits, workspace sized for the batch), then the
    oracle on the same prepared caches."""
    B, mx = len(lens), max(lens)
    torch.cuda.synchronize()
    hk = [bf16_to_u16(k) for k in kcs]
    hv = [bf16_to_u16(v) for v in vcs]
    want, wkc, wvc = oracle.decode_step(bf16_to_u16(q), bf16_to_u16(kn), bf16_to_u16(vn), hk, hv,
                                        lens, H, W.SCALE)
    kp = torch.tensor([t.data_ptr() for t in kcs], dtype=torch.int64, device="cuda")
    vp = torch.tensor([t.data_ptr() for t in vcs], dtype=torch.int64, device="cuda")
    lt = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = torch.zeros(lib.nc_decode_workspace_bytes(B, mx, H, 0), dtype=torch.uint8, device="cuda")
    out = torch.empty((B, ROW), dtype=torch.bfloat16, device="cuda")
    for call in range(2):  # the bench replays the step: counters must be back at zero
        st = lib.nc_decode_attention(_p(out), _p(q), _p(kn), _p(vn), _p(kp), _p(vp), _p(lt), B,
                                     H, W.SCALE, mx, 0, _p(ws), ws.numel(), _s())
        assert st == 0, lib.nc_status_string(st)
        torch.cuda.synchronize()
        assert_close_bf16(bf16_to_u16(out), want.reshape(B, ROW), what=f"{what} call {call}")
    for b, L in enumerate(lens):
        gk, gv = bf16_to_u16(kcs[b]), bf16_to_u16(vcs[b])
        assert ulp_diff_bf16(gk[L - 1], wkc[b][L - 1]).max() <= 1, f"{what}: appended K, seq {b}"
        assert np.array_equal(gv[L - 1], wvc[b][L - 1]), f"{what}: appended V, seq {b}"


def test_cfg1_pinned(lib):
    """cfg1: seed-0 Q/K/V, 511 cached keys normalised at positions 0..510, the new token at 511
    appended and attended to by the fused decode kernel."""
    q, kn, vn, kc, vc = W.cfg1_decode_case(seed=0)
    raw_rows = bf16_to_u16(kc[:W.CFG1_LEN - 1])
    q, kn, vn, kc, vc = (t.cuda() for t in (q, kn, vn, kc, vc))
    _normalise(lib, kc[:W.CFG1_LEN - 1], 0)
    torch.cuda.synchronize()
    # the bench's cache preparation agrees with the oracle's RoPE + QK-norm
    want_rows = oracle.apply_rope_rmsnorm(raw_rows, W.CFG1_LEN - 1, H, 0)
    assert ulp_diff_bf16(bf16_to_u16(kc[:W.CFG1_LEN - 1]), want_rows).max() <= 1
    _decode_and_check(lib, q, kn, vn, [kc], [vc], [W.CFG1_LEN], "cfg1")


def test_cfg2_pinned(lib):
    """cfg2: seed-1 Q/K/V through nc_rope_qknorm_append into an empty cache, then
    nc_flash_attention over all 2048 positions (the bench's step), end to end against the
    oracle's RoPE/QK-norm/append and attention on the raw inputs."""
    S = W.CFG2_SEQ
    q, k, v = W.cfg2_inputs(seed=1)
    hq, hk, hv = bf16_to_u16(q), bf16_to_u16(k), bf16_to_u16(v)
    z = np.zeros((S, H, D), np.uint16)
    wq, wkc, wvc = oracle.rope_qknorm_append(hq, hk, hv, z, z, S, H, 0)
    want = oracle.flash_attention(wq, wkc, wvc, S, S, H, W.SCALE, 0)
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    kc = torch.zeros((S, H, D), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.empty((S, ROW), dtype=torch.bfloat16, device="cuda")
    assert lib.nc_rope_qknorm_append(_p(dq), _p(dk), _p(dv), _p(kc), _p(vc), S, H, 0, _s()) == 0
    assert lib.nc_flash_attention(_p(out), _p(dq), _p(kc), _p(vc), S, S, H, W.SCALE, 0, _s()) == 0
    torch.cuda.synchronize()
    assert ulp_diff_bf16(bf16_to_u16(dq), wq).max() <= 1
    assert ulp_diff_bf16(bf16_to_u16(kc), wkc).max() <= 1
    assert np.array_equal(bf16_to_u16(vc), wvc)
    assert_close_bf16(bf16_to_u16(out), want, what="cfg2")


def test_cfg3_pinned_all_64(lib):
    """cfg3: all 64 sequences of the seed-2 kv_len draw (sum 63,344 keys) in one launch, as the
    bench times it (streaming layout, automatic split length)."""
    lens = W.cfg3_kv_lens()
    assert len(lens) == 64 and sum(lens) == 63344
    q, kn, vn, kcs, vcs = W.decode_batch_raw(lens, seed=2)
    for kc in kcs:
        _normalise(lib, kc, 0)
    _decode_and_check(lib, q, kn, vn, kcs, vcs, lens, "cfg3")


def test_cfg4_pinned(lib):
    """cfg4: 4 sequences, 1536 cached keys each (normalised at positions 0..1535), a seed-3 chunk
    of 512 appended per sequence, then one batched prefill launch over all four."""
    n, off, C = W.CFG4_BATCH, W.CFG4_OFFSET, W.CFG4_CHUNK
    rows = off + C
    q0, k0, v0 = W.cfg4_chunk_inputs()
    q, k, v = q0.cuda(), k0.cuda(), v0.cuda()
    kslab, vslab = W.cfg4_cache_raw(n, rows, seed=30)
    for i in range(n):
        _normalise(lib, kslab[i, :off], 0)
    torch.cuda.synchronize()
    hks, hvs = bf16_to_u16(kslab), bf16_to_u16(vslab)
    hq, hk, hv = bf16_to_u16(q0), bf16_to_u16(k0), bf16_to_u16(v0)
    wants, wqs, wks, wvs = [], [], [], []
    for i in range(n):
        wq, wkc, wvc = oracle.rope_qknorm_append(hq[i], hk[i], hv[i], hks[i], hvs[i], C, H, off)
        wants.append(oracle.flash_attention(wq, wkc, wvc, C, rows, H, W.SCALE, off))
        wqs.append(wq), wks.append(wkc), wvs.append(wvc)
    offs = torch.full((n,), off, dtype=torch.int32, device="cuda")
    out = torch.empty((n, C, ROW), dtype=torch.bfloat16, device="cuda")
    for i in range(n):
        assert lib.nc_rope_qknorm_append(_p(q[i]), _p(k[i]), _p(v[i]), _p(kslab[i]), _p(vslab[i]),
                                         C, H, off, _s()) == 0
    assert lib.nc_prefill_attention_batched(_p(out), _p(q), _p(kslab), _p(vslab), rows * ROW, rows,
                                            _p(offs), n, C, H, W.SCALE, _s()) == 0
    torch.cuda.synchronize()
    gks, gvs = bf16_to_u16(kslab), bf16_to_u16(vslab)
    for i in range(n):
        assert ulp_diff_bf16(bf16_to_u16(q[i]), wqs[i]).max() <= 1
        assert ulp_diff_bf16(gks[i][off:], wks[i][off:]).max() <= 1
        assert np.array_equal(gvs[i][off:], wvs[i][off:])
        assert_close_bf16(bf16_to_u16(out[i]), wants[i], what=f"cfg4 sequence {i}")

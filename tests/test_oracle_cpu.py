"""The CPU oracle against (a) an independent float64 numpy restatement of the reference's
math on small cases and (b) the golden vectors that the reference's own CUDA kernels produced
on a B200 (tests/golden/, made by tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

import oracle
from conftest import ROOT, assert_close_bf16, ulp_diff_bf16

H, D = 17, 128
SCALE = 1.0 / np.sqrt(128.0)
GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_kernels.npz")


def rand_u16(shape, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return oracle.f32_to_bf16_bits(rng.standard_normal(shape).astype(np.float32) * scale)


def np_rope_norm(x_u16, start_pos, norm=True):
    """float64 restatement of kernels/rope.cu:74-152 using the oracle's fp32 tables."""
    c, s = oracle.rope_tables()
    x = oracle.bf16_bits_to_f32(x_u16).astype(np.float64)
    S = x.shape[0]
    pos = np.arange(start_pos, start_pos + S)
    cc = c[pos][:, None, :].astype(np.float64)
    ss = s[pos][:, None, :].astype(np.float64)
    x0, x1 = x[..., :64], x[..., 64:]
    y = np.concatenate([x0 * cc + x1 * ss, -x0 * ss + x1 * cc], axis=-1)
    if norm:
        y = y / np.sqrt((y * y).mean(-1, keepdims=True) + 1e-6)
    return oracle.f32_to_bf16_bits(y.astype(np.float32))


def np_attention(q_u16, k_u16, v_u16, seq_q, kv_len, scale, off):
    q = oracle.bf16_bits_to_f32(q_u16).astype(np.float64).reshape(seq_q, H, D)
    k = oracle.bf16_bits_to_f32(k_u16).astype(np.float64).reshape(-1, H, D)[:kv_len]
    v = oracle.bf16_bits_to_f32(v_u16).astype(np.float64).reshape(-1, H, D)[:kv_len]
    s = np.einsum("qhd,khd->hqk", q, k) * scale
    qi = np.arange(seq_q)[:, None]
    kj = np.arange(kv_len)[None, :]
    mask = kj <= qi + off
    s = np.where(mask[None], s, -np.inf)
    m = s.max(-1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        p = np.exp(s - m)
        o = np.einsum("hqk,khd->qhd", p, v) / p.sum(-1)[..., None].transpose(1, 0, 2)
    return oracle.f32_to_bf16_bits(o.reshape(seq_q, H * D).astype(np.float32))


def test_rope_tables_shape_and_values():
    c, s = oracle.rope_tables()
    assert c.shape == (20480, 64) and s.shape == (20480, 64)
    assert np.all(c[0] == 1.0) and np.all(s[0] == 0.0)
    # frequency 0 is 1 rad per position; fp32 angles are exact for small positions
    np.testing.assert_allclose(c[:100, 0], np.cos(np.arange(100, dtype=np.float32)), atol=1e-6)
    np.testing.assert_allclose(s[:100, 0], np.sin(np.arange(100, dtype=np.float32)), atol=1e-6)
    assert np.all(np.abs(c * c + s * s - 1.0) < 1e-5)


@pytest.mark.parametrize("seq_len,start_pos", [(1, 0), (5, 511), (40, 2000), (3, 20477)])
def test_oracle_rope_rmsnorm_vs_numpy(seq_len, start_pos):
    x = rand_u16((seq_len, H, D), seq_len + start_pos)
    got = oracle.apply_rope_rmsnorm(x, seq_len, H, start_pos)
    want = np_rope_norm(x, start_pos)
    assert ulp_diff_bf16(got, want).max() <= 1
    got_r = oracle.apply_rope(x, seq_len, H, start_pos)
    want_r = np_rope_norm(x, start_pos, norm=False)
    assert ulp_diff_bf16(got_r, want_r).max() <= 1


@pytest.mark.parametrize("seq_q,kv_len,off", [(1, 1, 0), (1, 37, 36), (5, 5, 0), (9, 40, 31),
                                              (33, 33, 0), (4, 10, 100), (6, 6, -3)])
def test_oracle_attention_vs_numpy(seq_q, kv_len, off):
    q = rand_u16((seq_q, H, D), 1)
    k = rand_u16((kv_len, H, D), 2)
    v = rand_u16((kv_len, H, D), 3)
    got = oracle.flash_attention(q, k, v, seq_q, kv_len, H, SCALE, off)
    want = np_attention(q, k, v, seq_q, kv_len, SCALE, off)
    assert_close_bf16(got, want, max_abs=4e-3, mean_abs=2e-4, what="oracle vs float64")


def test_oracle_decode_step_is_append_then_attend():
    lens = [1, 7, 30]
    rows = 40
    q = rand_u16((3, H, D), 10)
    kn = rand_u16((3, H, D), 11)
    vn = rand_u16((3, H, D), 12)
    kcs = [rand_u16((rows, H, D), 20 + b) for b in range(3)]
    vcs = [rand_u16((rows, H, D), 30 + b) for b in range(3)]
    out, kc2, vc2 = oracle.decode_step(q, kn, vn, kcs, vcs, lens, H, SCALE)
    for b, L in enumerate(lens):
        qn, kc, vc = oracle.rope_qknorm_append(q[b:b + 1], kn[b:b + 1], vn[b:b + 1], kcs[b], vcs[b],
                                               1, H, L - 1)
        assert np.array_equal(kc, kc2[b]) and np.array_equal(vc, vc2[b])
        o = oracle.flash_attention(qn, kc, vc, 1, L, H, SCALE, L - 1)
        assert np.array_equal(o[0], out[b])


# ------------------------------------------------------------------------ golden vectors
def _golden():
    if not os.path.exists(GOLDEN):
        pytest.fail(f"missing golden vectors {GOLDEN} (tests/golden/make_golden.py on a GPU box)")
    return np.load(GOLDEN)


def test_golden_rope_table_bit_exact():
    g = _golden()
    c, s = oracle.rope_tables()
    idx = g["table_positions"]
    assert np.array_equal(g["table_cos"].view(np.uint32), c[idx].view(np.uint32))
    assert np.array_equal(g["table_sin"].view(np.uint32), s[idx].view(np.uint32))


def test_golden_rope():
    g = _golden()
    for name in ("rope", "rope_rmsnorm"):
        x = g[f"{name}_in"]
        seq_len, start = (int(v) for v in g[f"{name}_args"])
        fn = oracle.apply_rope if name == "rope" else oracle.apply_rope_rmsnorm
        got = fn(x, seq_len, H, start)
        d = ulp_diff_bf16(got, g[f"{name}_out"])
        assert d.max() <= 1, name
        assert (d == 0).mean() >= 0.99, name


def test_golden_attention():
    g = _golden()
    names = [n[:-5] for n in g.files if n.startswith("attn_") and n.endswith("_args")]
    assert len(names) >= 5
    for n in names:
        seq_q, kv_len, off = (int(v) for v in g[n + "_args"])
        got = oracle.flash_attention(g[n + "_q"], g[n + "_k"], g[n + "_v"], seq_q, kv_len, H,
                                     SCALE, off)
        assert_close_bf16(got, g[n + "_out"], what=n)


# ------------------------------------------------------------------------------ sampling
def _sample_intervals(row_u16, T, k, p):
    """Engine::sample's kept entries and their renormalised running sums, in float64 (for
    checking the oracle's choices away from the interval edges)."""
    lf = oracle.bf16_bits_to_f32(row_u16).astype(np.float64)
    pr = np.exp((lf - lf.max()) / T)
    pr /= pr.sum()
    order = sorted(range(len(pr)), key=lambda i: (-pr[i], i))
    if 0 < k < len(pr):
        order = order[:k]
    if p < 1.0:
        cs = np.cumsum(pr[order])
        cut = int(np.argmax(cs > p)) + 1 if (cs > p).any() else len(order)
        order = order[:cut]
    w = pr[order] / pr[order].sum()
    return order, np.cumsum(w)


def test_oracle_sample_matches_intervals():
    """orc_sample (Engine::sample, src/engine.cpp:88-131): greedy at temperature 0 is the first
    maximum; otherwise the draw r picks the entry whose renormalised running-sum interval holds
    r (checked at interval midpoints, away from fp32 rounding)."""
    rng = np.random.default_rng(11)
    V = 4096
    row = oracle.f32_to_bf16_bits((rng.standard_normal(V) * 2.0).astype(np.float32))
    row[[17, 900]] = oracle.f32_to_bf16_bits(np.array([9.0, 9.0], np.float32))  # tied maxima
    assert oracle.sample(row, 0.0, 50, 0.9, 0.5) == 17
    for T, k, p in [(1.0, 50, 0.9), (0.7, 5, 1.0), (1.5, 200, 0.5), (1.0, 1, 0.9)]:
        order, cs = _sample_intervals(row, T, k, p)
        lo = np.concatenate([[0.0], cs[:-1]])
        for j in range(len(order)):
            r = 0.5 * (lo[j] + cs[j])
            if cs[j] - lo[j] < 1e-5:
                continue
            assert oracle.sample(row, T, k, p, r) == order[j], (T, k, p, j)
    # top_k == 1: always the first maximum
    assert oracle.sample(row, 1.0, 1, 1.0, 0.999) == 17

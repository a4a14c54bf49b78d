"""Skinny tcgen05 GEMM of the decode step (nc_gemm_skinny) against a torch fp32 reference.

The reference computes gemm_half in fp32 accumulation with one bf16 rounding
(kernels/gemm.cu:62-113; gemm_half_residual adds the residual before that rounding,
kernels/gemm.cu:115-166).  Checks: plain products over the batch sizes and shapes of the decode
call sites (src/model.cpp:114-116, :139, :149-153, :174) plus ragged N and K tails; each fused
step (RMSNorm row scale, residual, in-place residual, ReLU^2, tanh cap, segmented Q|K|V output);
fixed-order split-K through a thread-block cluster (bit-identical repeats, CUDA-graph replay
equal to eager, explicit split counts agreeing); and chains of dependent calls launched with
programmatic dependent launch.  Also the two passes at the ends of a decode step: the embedding
gather + RMSNorm and the on-device first-maximum argmax.

Tolerance.  The tensor cores' fp32 accumulation is not exact fp32 summation: measured on B200
against an fp64 product, cuBLAS's bf16 GEMM (torch.matmul) and this kernel without a K split
give identical error statistics, up to 4.5e-4 x sum_k |x_k w_k| (and a K split only lowers the
error).  So a result must be within one bf16 ulp of the fp64 product plus 1e-3 x that sum.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

NORM_EPS = 1e-6


@pytest.fixture(scope="module")
def G():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc

    yield nc.gemm
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) == 0, "a kernel's bounded wait gave up"


def rnd(shape, seed, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * std).to(torch.bfloat16)


def ref_product(x, w):
    return (x.double() @ w.double().t()).float()


def accum_slack(x, w, scale=None):
    """1e-3 x sum_k |x_k w_k| per output (times the row scale when the row is scaled)."""
    mag = (x.double().abs() @ w.double().abs().t()).float() * 1e-3
    return mag if scale is None else mag * scale


def assert_ulp(got, want_f32, what, slack=0.0):
    """got (bf16) against an fp32 result: within one bf16 ulp of it plus `slack`."""
    want = want_f32.float()
    d = (got.float() - want).abs()
    bound = want.abs() * 2.0 ** -7 + 1e-6 + slack
    bad = d > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {d.numel()} beyond the bound, "
                           f"max |d| {d.max().item():.3g}")


@pytest.mark.parametrize("M", [1, 4, 8, 16, 17, 32, 33, 64])
@pytest.mark.parametrize("N,K", [(2176, 2176), (8704, 2176), (2176, 8704)])
def test_plain_product(G, M, N, K):
    x, w = rnd((M, K), 1), rnd((N, K), 2, 0.02)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm_skinny(out, x, w)
    torch.cuda.synchronize()
    assert_ulp(out, ref_product(x, w), f"M={M} N={N} K={K}", accum_slack(x, w))


@pytest.mark.parametrize("M,N,K", [(8, 200, 136), (3, 130, 72), (8, 65536, 2176),
                                   (5, 6528, 2176), (2, 128, 8)])
def test_ragged_and_large_shapes(G, M, N, K):
    x, w = rnd((M, K), 3), rnd((N, K), 4, 0.05)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm_skinny(out, x, w)
    torch.cuda.synchronize()
    assert_ulp(out, ref_product(x, w), f"M={M} N={N} K={K}", accum_slack(x, w))


@pytest.mark.parametrize("M", [1, 8, 40])
def test_norm_input(G, M):
    """NC_GEMM_NORM_INPUT: the product of RMSNorm(x) (kernels/rmsnorm.cu) with w.  Compared
    with r_m * (x @ w^T) in fp32 (one ulp); the reference's own order, which rounds RMSNorm(x)
    to bf16 before the GEMM, differs from that by the rounding of the normalised input, so it
    gets the model tolerance (max 2e-2, mean 2e-3 absolute)."""
    N, K = 8704, 2176
    x, w = rnd((M, K), 7, 3.0), rnd((N, K), 8, 0.02)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm_skinny(out, x, w, flags=G.NORM_INPUT)
    torch.cuda.synchronize()
    xf = x.float()
    r = torch.rsqrt(xf.square().sum(-1, keepdim=True) / K + NORM_EPS)
    assert_ulp(out, r * ref_product(x, w), f"norm M={M}", accum_slack(x, w, r))
    # Reference order: RMSNorm(x) rounded to bf16 (relative error <= 2^-9 per element), then
    # the GEMM: within one ulp, the accumulation slack and 2^-9 x sum_k |xn_k w_k|.
    xn = (xf * r).to(torch.bfloat16)
    want = ref_product(xn, w)
    d = (out.float() - want).abs()
    bound = want.abs() * 2.0 ** -7 + 1e-6 + accum_slack(x, w, r) * (1 + 2.0 ** -9 / 1e-3)
    assert (d <= bound).all() and d.mean() <= 2e-3


def test_residual_and_in_place(G):
    M, N, K = 8, 2176, 8704
    x, w, res = rnd((M, K), 9), rnd((N, K), 10, 0.02), rnd((M, N), 11)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm_skinny(out, x, w, residual=res)
    acc = res.clone()
    G.gemm_half_residual(acc, x, w, acc, M, N, K)  # in place, as src/model.cpp:139
    torch.cuda.synchronize()
    want = ref_product(x, w) + res.float()
    assert_ulp(out, want, "residual", accum_slack(x, w))
    assert torch.equal(acc, out)


def test_relu2(G):
    """NC_GEMM_RELU2 after NORM_INPUT: the MLP up projection (src/model.cpp:149-150)."""
    M, N, K = 8, 8704, 2176
    x, w = rnd((M, K), 12), rnd((N, K), 13, 0.02)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm_skinny(out, x, w, flags=G.NORM_INPUT | G.RELU2)
    torch.cuda.synchronize()
    xf = x.float()
    r = torch.rsqrt(xf.square().sum(-1, keepdim=True) / K + NORM_EPS)
    # relu(v)^2 amplifies v's rounding by 2|v|: compare at two ulps of the squared value.
    v = r * ref_product(x, w)
    want = torch.relu(v).square()
    d = (out.float() - want).abs()
    assert (d <= want.abs() * 2.0 ** -6 + 1e-6 + 3 * v.abs() * accum_slack(x, w, r)).all()
    assert int((out.float() == 0).sum()) > M * N // 3  # roughly half the products are < 0


def test_tanh_cap_lm_head(G):
    """NC_GEMM_NORM_INPUT | NC_GEMM_TANH_CAP: final norm, LM head and soft cap 15
    (src/model.cpp:170-177) over the full 65536-row vocabulary."""
    M, N, K, cap = 8, 65536, 2176, 15.0
    x, w = rnd((M, K), 14), rnd((N, K), 15, 0.5)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm_skinny(out, x, w, flags=G.NORM_INPUT | G.TANH_CAP, cap=cap)
    torch.cuda.synchronize()
    xf = x.float()
    r = torch.rsqrt(xf.square().sum(-1, keepdim=True) / K + NORM_EPS)
    want = cap * torch.tanh(r * ref_product(x, w) / cap)
    assert want.abs().max() > 10.0  # the cap is exercised
    d = (out.float() - want).abs()  # d tanh <= 1: the product's slack carries over
    assert (d <= want.abs() * 2.0 ** -7 + 1e-4 + accum_slack(x, w, r)).all(), d.max()


def test_segmented_qkv(G):
    """A fused [q; k; v] weight with seg_cols = 2176 writes three [M, 2176] arrays: the three
    projections of src/model.cpp:114-116 in one pass over the weights."""
    M, D, K = 8, 2176, 2176
    x = rnd((M, K), 16)
    wq, wk, wv = rnd((D, K), 17, 0.02), rnd((D, K), 18, 0.02), rnd((D, K), 19, 0.02)
    w = torch.cat([wq, wk, wv], 0)
    out = torch.empty((3, M, D), dtype=torch.bfloat16, device="cuda")
    G.gemm_skinny(out, x, w, flags=G.NORM_INPUT, seg_cols=D)
    torch.cuda.synchronize()
    xf = x.float()
    r = torch.rsqrt(xf.square().sum(-1, keepdim=True) / K + NORM_EPS)
    for i, wi in enumerate((wq, wk, wv)):
        assert_ulp(out[i], r * ref_product(x, wi), f"segment {i}", accum_slack(x, wi, r))


def test_split_k_deterministic_and_graph(G):
    """Fixed-order split-K: repeats are bit-identical, a CUDA-graph replay equals the eager
    call, and explicit split counts (1 to 12, 16 and 136 clamped to 12) all meet the bound."""
    M, N, K = 8, 2176, 8704
    x, w, res = rnd((M, K), 20), rnd((N, K), 21, 0.02), rnd((M, N), 22)
    outs = []
    for _ in range(3):
        o = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        G.gemm_skinny(o, x, w, residual=res)
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    g_out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            G.gemm_skinny(g_out, x, w, residual=res)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        g_out.zero_()
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(g_out, outs[0])
    want = ref_product(x, w) + res.float()
    for splits in (1, 2, 3, 5, 7, 8, 12, 16, 136):
        o = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        G.gemm_skinny(o, x, w, residual=res, splits=splits)
        torch.cuda.synchronize()
        assert_ulp(o, want, f"splits={splits}", accum_slack(x, w))
    del graph


def test_chain_of_dependent_calls(G):
    """Back-to-back calls where each consumes the previous output (the decode step's
    O -> up -> down chain, launched with programmatic dependent launch: each call streams
    its first weight boxes before the previous one has finished) give the results of the same
    calls separated by synchronizations."""
    M, D, H = 8, 2176, 8704
    x = rnd((M, D), 23)
    a = rnd((M, D), 24)
    wo, wu, wd = rnd((D, D), 25, 0.02), rnd((H, D), 26, 0.02), rnd((D, H), 27, 0.02)
    xs = x.clone()
    h = torch.empty((M, H), dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        G.gemm_skinny(xs, a, wo, residual=xs)
        G.gemm_skinny(h, xs, wu, flags=G.NORM_INPUT | G.RELU2)
        G.gemm_skinny(xs, h, wd, residual=xs)
    torch.cuda.synchronize()
    # same chain one call at a time with a synchronize between calls
    xr = x.clone()
    hr = torch.empty_like(h)
    for _ in range(2):
        G.gemm_skinny(xr, a, wo, residual=xr)
        torch.cuda.synchronize()
        G.gemm_skinny(hr, xr, wu, flags=G.NORM_INPUT | G.RELU2)
        torch.cuda.synchronize()
        G.gemm_skinny(xr, hr, wd, residual=xr)
        torch.cuda.synchronize()
    assert torch.equal(xs, xr) and torch.equal(h, hr)


# ----------------------------------------------------------------------- ends of a decode step
def test_embed_rmsnorm(G):
    """nc_embed_rmsnorm against the reference's two passes (kernels/ops.cu:9-20 gather, then
    kernels/rmsnorm.cu: x * rsqrt(sum(x^2)/n + 1e-6), one bf16 rounding) computed in fp64:
    within one bf16 ulp.  Repeated and out-of-range token ids included."""
    import nanochat_inferonly_lightning_b200 as nc

    V, Dm = 65536, 2176
    table = rnd((V, Dm), 30, 0.7)
    tokens = torch.tensor([0, 5, 65535, 5, 12345, 777, 1, 40000], dtype=torch.int32,
                          device="cuda")
    out = torch.empty((8, Dm), dtype=torch.bfloat16, device="cuda")
    G.embed_rmsnorm(out, table, tokens)
    torch.cuda.synchronize()
    rows = table[tokens.long()].double()
    want = rows * torch.rsqrt(rows.square().sum(-1, keepdim=True) / Dm + NORM_EPS)
    d = (out.double() - want).abs()
    assert (d <= want.abs() * 2.0 ** -8 + 1e-6).all(), d.max()
    assert torch.equal(out[1], out[3])
    assert nc.device_status(reset=True) == 0
    bad = torch.tensor([3, -1, V], dtype=torch.int32, device="cuda")
    out3 = torch.full((3, Dm), 1.0, dtype=torch.bfloat16, device="cuda")
    G.embed_rmsnorm(out3, table, bad)
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) == 0x800  # range check flagged, no out-of-bounds read
    assert int(out3[1:].count_nonzero()) == 0 and int(out3[0].count_nonzero()) > 0


def test_argmax_rows_first_maximum(G):
    """nc_argmax_rows: the first maximum of each row (src/engine.cpp:88-95, strict '>'), with
    ties planted at several distances (same thread, same warp, other warps, first and last
    column) and rows that are constant."""
    R, C = 12, 65536
    logits = rnd((R, C), 31, 3.0)
    top = 40.0
    plants = {0: [7, 3], 1: [100, 9000], 2: [65535, 0], 3: [8191, 8192], 4: [64000, 64001],
              5: [12, 13, 14], 6: [70, 30000, 65000], 7: [65535]}
    for r, cols in plants.items():
        for c in cols:
            logits[r, c] = top
    logits[8] = 1.5  # constant row: index 0
    logits[9, :] = -2.0
    logits[9, 4097] = -1.0
    out = torch.empty(R, dtype=torch.int32, device="cuda")
    G.argmax_rows(out, logits)
    torch.cuda.synchronize()
    want = torch.argmax(logits.float(), dim=-1)  # first occurrence of the maximum
    assert torch.equal(out.long(), want)
    assert int(out[0]) == 3 and int(out[2]) == 0 and int(out[8]) == 0 and int(out[9]) == 4097


def _sample_margin(row_f32, T, k, p, r):
    """Distance (float64) from the draw r and from top_p to the nearest running-sum edge of
    Engine::sample's intervals: below ~1e-5 fp32 summation order can move the choice."""
    lf = row_f32.astype(np.float64)
    pr = np.exp((lf - lf.max()) / T)
    pr /= pr.sum()
    if 0 < k < len(pr):
        order = np.lexsort((np.arange(len(pr)), -pr))[:k]
    elif p < 1.0:  # top-p alone sorts the whole row
        order = np.lexsort((np.arange(len(pr)), -pr))
    else:  # no filter: index order
        order = np.arange(len(pr))
    cs = np.cumsum(pr[order])
    m = np.abs(cs - p).min() if p < 1.0 else 1.0
    if p < 1.0 and (cs > p).any():
        order = order[:int(np.argmax(cs > p)) + 1]
    w = np.cumsum(pr[order] / pr[order].sum())
    return min(m, np.abs(w - r).min())


def test_sample_rows_against_oracle(G):
    """nc_sample_rows against orc_sample (Engine::sample, src/engine.cpp:62-131, with the draw
    given) on 64 rows of 65536 bf16 logits: several temperatures, top-k from 1 to 1024, top-p
    on and off, rows with tied values.  Every row whose draw and top-p lie more than 1e-4 from
    an interval edge must give the oracle's token; at most a few rows are that close."""
    import numpy as np
    import oracle

    R, V = 64, 65536
    g = torch.Generator(device="cuda").manual_seed(40)
    logits = (torch.randn((R, V), generator=g, device="cuda") * 2.5).to(torch.bfloat16)
    logits[5, 1000:1100] = 9.0   # a block of tied maxima
    logits[6, ::7] = 4.0         # many ties inside the top-k
    u = torch.rand(R, generator=g, device="cuda")
    host = oracle.f32_to_bf16_bits(logits.float().cpu().numpy())
    uh = u.cpu().numpy()
    cases = [(1.0, 50, 0.9), (0.7, 50, 1.0), (1.3, 1024, 0.95), (0.5, 1, 0.9), (2.0, 300, 0.5)]
    skipped = 0
    for T, k, p in cases:
        out = torch.empty(R, dtype=torch.int32, device="cuda")
        G.sample_rows(out, logits, T, k, p, u)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for r in range(R):
            want = oracle.sample(host[r], T, k, p, float(uh[r]))
            if got[r] != want:
                lf = oracle.bf16_bits_to_f32(host[r])
                assert _sample_margin(lf, T, k, p, float(uh[r])) < 1e-4, (T, k, p, r, got[r], want)
                skipped += 1
    assert skipped <= 3, skipped
    # top_k off (0, or >= vocab) with top_p off: the whole row in index order.  Its 65536
    # intervals are ~1.5e-5 wide, as wide as the gap between a sequential and a parallel fp32
    # running sum, so the draw is checked against exact (fp64) running sums: the chosen index's
    # interval must lie within 1e-4 of r.
    for T, k in [(1.0, 0), (0.8, V)]:
        out = torch.empty(R, dtype=torch.int32, device="cuda")
        G.sample_rows(out, logits, T, k, 1.0, u)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for r in range(R):
            lf = oracle.bf16_bits_to_f32(host[r]).astype(np.float64)
            w = np.exp((lf - lf.max()) / T)
            cs = np.cumsum(w / w.sum())
            lo = cs[got[r] - 1] if got[r] > 0 else 0.0
            assert lo - 1e-4 <= uh[r] <= cs[got[r]] + 1e-4, (T, k, r, got[r])
    # top-p over the whole row (top_k off).  The kept prefix can hold thousands of entries with
    # intervals ~1e-5 wide, so the check is against exact (fp64) sums over the row sorted as
    # the reference sorts it (descending probability, ties by ascending index): the chosen index
    # must lie in the prefix whose running sum first exceeds top_p (within 1e-4 of the edge),
    # and its renormalised interval must lie within 1e-4 of r.  Rows where the peaked
    # distribution leaves wide intervals must give the oracle's token exactly.  Row 7 is made
    # constant: all 65536 entries share one key (the case a 16-bit per-key count cannot hold).
    lg = logits.clone()
    lg[7] = 1.5
    host_p = oracle.f32_to_bf16_bits(lg.float().cpu().numpy())
    exact_rows = 0
    for T, k, p in [(1.0, 0, 0.9), (0.6, 0, 0.5), (2.0, V, 0.95), (0.3, 0, 0.99)]:
        out = torch.empty(R, dtype=torch.int32, device="cuda")
        G.sample_rows(out, lg, T, k, p, u)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for r in range(R):
            lf = oracle.bf16_bits_to_f32(host_p[r]).astype(np.float64)
            pr = np.exp((lf - lf.max()) / T)
            pr /= pr.sum()
            order = np.lexsort((np.arange(V), -pr))
            cs = np.cumsum(pr[order])
            pos = int(np.nonzero(order == got[r])[0][0])
            cut = int(np.argmax(cs > p)) + 1 if (cs > p).any() else V
            assert pos < cut or cs[pos - 1] <= p + 1e-4, (T, k, p, r, pos, cut)
            s2 = cs[cut - 1]
            lo = cs[pos - 1] / s2 if pos > 0 else 0.0
            hi = cs[pos] / s2
            assert lo - 1e-4 <= uh[r] <= hi + 1e-4, (T, k, p, r, got[r], lo, hi, uh[r])
            if _sample_margin(oracle.bf16_bits_to_f32(host_p[r]), T, k, p, float(uh[r])) > 1e-4:
                assert got[r] == oracle.sample(host_p[r], T, k, p, float(uh[r])), (T, k, p, r)
                exact_rows += 1
    assert exact_rows >= R // 2, exact_rows
    # temperature 0 is the greedy path
    out = torch.empty(R, dtype=torch.int32, device="cuda")
    G.sample_rows(out, logits, 0.0, 50, 0.9, None)
    torch.cuda.synchronize()
    assert torch.equal(out.long(), torch.argmax(logits.float(), dim=-1))

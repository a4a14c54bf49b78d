"""Prompt-pass tcgen05 GEMM (nc_gemm) against an fp64 product, with the tolerance and helpers of
the decode-step GEMM tests (tests/test_gpu_gemm.py): one bf16 ulp of the exact product plus
1e-3 x sum_k |x_k w_k| for the tensor cores' fp32 accumulation.

Shapes: the prompt call sites of src/model.cpp:114-116, :139, :149-150, :153 at 8 x 256 prompt
tokens (M = 2048) and at other row counts, including M and N that are not multiples of the
128 x 256 tile and K that is not a multiple of the 64-wide K block; each fused step (RMSNorm row
scale, residual in place, ReLU^2, tanh cap, segmented Q|K|V output); repeat determinism; and
agreement with the decode-step kernel where both apply (M <= 64).
"""
import pytest

from test_gpu_gemm import NORM_EPS, accum_slack, assert_ulp, ref_product, rnd

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def G():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc

    yield nc.gemm
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) == 0, "a kernel's bounded wait gave up"


def rscale(x):
    xf = x.float()
    return torch.rsqrt(xf.square().sum(-1, keepdim=True) / x.shape[1] + NORM_EPS)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (37, 264, 136), (128, 256, 2176),
                                   (300, 2176, 2176), (2048, 2176, 8704), (1000, 8704, 2176),
                                   (2048, 6528, 2176), (129, 520, 72)])
def test_tile_product(G, M, N, K):
    x, w = rnd((M, K), M + 1), rnd((N, K), N + K, 0.02)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm(out, x, w)
    torch.cuda.synchronize()
    assert_ulp(out, ref_product(x, w), f"M={M} N={N} K={K}", accum_slack(x, w))


def test_tile_qkv_segmented_with_norm(G):
    """Fused [q; k; v] weight, RMSNorm row scale, three [M, 2176] outputs (src/model.cpp:110-116
    for a 2048-token prompt pass)."""
    M, D, K = 2048, 2176, 2176
    x = rnd((M, K), 21, 3.0)
    ws = [rnd((D, K), 22 + i, 0.02) for i in range(3)]
    out = torch.empty((3, M, D), dtype=torch.bfloat16, device="cuda")
    G.gemm(out, x, torch.cat(ws, 0), flags=G.NORM_INPUT, seg_cols=D)
    torch.cuda.synchronize()
    r = rscale(x)
    for i, wi in enumerate(ws):
        assert_ulp(out[i], r * ref_product(x, wi), f"segment {i}", accum_slack(x, wi, r))


def test_tile_residual_in_place(G):
    """Output projection / MLP down projection + residual, in place (src/model.cpp:139, :153)."""
    M, N, K = 700, 2176, 8704
    x, w, res = rnd((M, K), 31), rnd((N, K), 32, 0.02), rnd((M, N), 33)
    acc = res.clone()
    G.gemm(acc, x, w, residual=acc)
    torch.cuda.synchronize()
    assert_ulp(acc, ref_product(x, w) + res.float(), "residual in place", accum_slack(x, w))


def test_tile_norm_relu2(G):
    """MLP up projection with RMSNorm and ReLU^2 (src/model.cpp:146-150)."""
    M, N, K = 513, 8704, 2176
    x, w = rnd((M, K), 41), rnd((N, K), 42, 0.02)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm(out, x, w, flags=G.NORM_INPUT | G.RELU2)
    torch.cuda.synchronize()
    r = rscale(x)
    v = r * ref_product(x, w)
    want = torch.relu(v).square()
    d = (out.float() - want).abs()
    assert (d <= want.abs() * 2.0 ** -6 + 1e-6 + 3 * v.abs() * accum_slack(x, w, r)).all()


def test_tile_tanh_cap(G):
    M, N, K, cap = 200, 4096, 2176, 15.0
    x, w = rnd((M, K), 51), rnd((N, K), 52, 0.5)
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    G.gemm(out, x, w, flags=G.NORM_INPUT | G.TANH_CAP, cap=cap)
    torch.cuda.synchronize()
    r = rscale(x)
    want = cap * torch.tanh(r * ref_product(x, w) / cap)
    assert want.abs().max() > 10.0
    d = (out.float() - want).abs()
    assert (d <= want.abs() * 2.0 ** -7 + 1e-4 + accum_slack(x, w, r)).all(), d.max()


def test_tile_deterministic_and_matches_skinny(G):
    """Repeats are bit-identical; at M <= 64 the result meets the same bound as the decode-step
    kernel's (both are checked against the fp64 product)."""
    M, N, K = 48, 2176, 2176
    x, w = rnd((M, K), 61), rnd((N, K), 62, 0.02)
    a = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    s = torch.empty_like(a)
    G.gemm(a, x, w, flags=G.NORM_INPUT)
    G.gemm(b, x, w, flags=G.NORM_INPUT)
    G.gemm_skinny(s, x, w, flags=G.NORM_INPUT)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    r = rscale(x)
    assert_ulp(a, r * ref_product(x, w), "tile", accum_slack(x, w, r))
    assert_ulp(s, r * ref_product(x, w), "skinny", accum_slack(x, w, r))


def test_tile_rejects_bad_shapes(G):
    x = torch.zeros((8, 64), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((12, 64), dtype=torch.bfloat16, device="cuda")  # N % 8 != 0
    out = torch.zeros((8, 12), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        G.gemm(out, x, w)

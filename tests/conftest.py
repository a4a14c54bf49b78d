import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_libraries():
    """Builds the product library and the C oracle if they are missing or stale (nvcc
    cross-compiles without a GPU); the reference-kernel rebuild only where the reference tree
    exists."""
    from nanochat_inferonly_lightning_b200 import build as pkg_build
    from oracle import build as orc_build
    from oracle import build_ref

    pkg_build.build(verbose=False)
    orc_build.build(verbose=False)
    build_ref.build(verbose=False)
    build_ref.build_model(verbose=False)
    yield


def bf16_to_u16(t):
    """torch bf16 tensor -> numpy uint16 bit patterns (CPU copy)."""
    import torch

    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)


def u16_to_bf16(a, device="cpu"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def assert_close_bf16(got_u16, want_u16, max_abs=2e-2, mean_abs=2e-3, what=""):
    """The north-star tolerance on bf16 outputs: max-abs 2e-2 and mean-abs 2e-3; NaN positions
    must agree exactly."""
    from oracle import bf16_bits_to_f32

    g = bf16_bits_to_f32(got_u16).astype(np.float64)
    w = bf16_bits_to_f32(want_u16).astype(np.float64)
    gn, wn = np.isnan(g), np.isnan(w)
    assert np.array_equal(gn, wn), f"{what}: NaN positions differ ({gn.sum()} vs {wn.sum()})"
    ok = ~wn
    if not ok.any():
        return 0.0, 0.0
    d = np.abs(g[ok] - w[ok])
    mx, mn = float(d.max()), float(d.mean())
    assert mx <= max_abs, f"{what}: max-abs {mx:.3e} > {max_abs}"
    assert mn <= mean_abs, f"{what}: mean-abs {mn:.3e} > {mean_abs}"
    return mx, mn


def ulp_diff_bf16(a_u16, b_u16):
    """Distance in bf16 units-in-the-last-place between two bit-pattern arrays (finite)."""
    a = np.asarray(a_u16, np.uint16).astype(np.int32)
    b = np.asarray(b_u16, np.uint16).astype(np.int32)
    # map sign-magnitude to a monotone integer line
    a = np.where(a & 0x8000, -(a & 0x7FFF), a)
    b = np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(a - b)

"""nc_decode_attention_noalloc: the decode entry point that allocates no device memory.

It serves callers that cannot hand the library a workspace (device memory planned by an
outside allocator, host bindings without a device allocator, latency-critical loops that
must not call cudaMalloc).  Checked here through the C ABI against the regular entry point,
nc_decode_attention with a caller-provided workspace, on two calls in a row (the shared
in-library scratch must leave its split counters ready for the next call).  Runs last in the
suite (file name) and stands alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from conftest import assert_close_bf16, bf16_to_u16

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H, D = 17, 128
SCALE = 1.0 / np.sqrt(128.0)


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _batch(lens, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows = max(lens) + 3

    def rnd(*shape):
        return torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)

    q, kn, vn = rnd(len(lens), H, D), rnd(len(lens), H, D), rnd(len(lens), H, D)
    kcs = [rnd(rows, H, D) for _ in lens]
    vcs = [rnd(rows, H, D) for _ in lens]
    return q, kn, vn, kcs, vcs


def _ptr_table(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")


@pytest.mark.parametrize("lens", [[1, 17, 300, 2048], [5] * 3 + [4000], [129] * 64])
def test_noalloc_matches_workspace_entry_point(lens):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc

    lib = nc.load()
    B, mx = len(lens), max(lens)
    q, kn, vn, kcs, vcs = _batch(lens, seed=len(lens) + mx)
    lt = torch.tensor(lens, dtype=torch.int32, device="cuda")

    # regular entry point, caller workspace, on its own copy of the caches
    k_ref = [k.clone() for k in kcs]
    v_ref = [v.clone() for v in vcs]
    ws = torch.zeros(lib.nc_decode_workspace_bytes(B, mx, H, 0), dtype=torch.uint8, device="cuda")
    out_ref = torch.empty((B, H * D), dtype=torch.bfloat16, device="cuda")
    assert lib.nc_decode_attention(_p(out_ref), _p(q), _p(kn), _p(vn), _p(_ptr_table(k_ref)),
                                   _p(_ptr_table(v_ref)), _p(lt), B, H, SCALE, mx, 0, _p(ws),
                                   ws.numel(), _stream()) == 0
    torch.cuda.synchronize()
    want = bf16_to_u16(out_ref)

    # allocation-free entry point, twice in a row on the same caches
    kt, vt = _ptr_table(kcs), _ptr_table(vcs)
    for call in range(2):
        out = torch.full((B, H * D), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = lib.nc_decode_attention_noalloc(_p(out), _p(q), _p(kn), _p(vn), _p(kt), _p(vt),
                                             _p(lt), B, H, SCALE, mx, _stream())
        assert st == 0, lib.nc_status_string(st)
        torch.cuda.synchronize()
        assert_close_bf16(bf16_to_u16(out), want, what=f"noalloc call {call} lens={lens[:4]}")
    # the appended key/value rows agree with the regular entry point's
    for b in range(B):
        assert torch.equal(kcs[b], k_ref[b]) and torch.equal(vcs[b], v_ref[b])
    assert nc.device_status(reset=True) == 0


def test_noalloc_rejects_beyond_its_limits():
    import nanochat_inferonly_lightning_b200 as nc

    lib = nc.load()
    P = ctypes.c_void_p
    # batch above 256 and kv_len above the RoPE table are refused before any device work
    assert lib.nc_decode_attention_noalloc(P(256), P(256), None, None, P(256), P(256), P(256),
                                           257, H, SCALE, 128, None) == 7
    assert lib.nc_decode_attention_noalloc(P(256), P(256), None, None, P(256), P(256), P(256),
                                           4, H, SCALE, 20481, None) == 7

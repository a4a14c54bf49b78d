"""nc_decode_attention_noalloc: the decode entry point that allocates no device memory.

It serves callers that cannot hand the library a workspace (device memory planned by an
outside allocator, host bindings without a device allocator, latency-critical loops that
must not call cudaMalloc).  Checked here through the C ABI against the regular entry point,
nc_decode_attention with a caller-provided workspace, on two calls in a row (the shared
in-library scratch must be ready for the next call), and against the CPU oracle on the same
inputs.  Cases cover one sequence (one split and many), the largest batch with long caches
(where the split length has to grow to fit the fixed array), and a length above max_kv_len
(clamped and flagged).  Runs last in the suite (file name) and stands alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import assert_close_bf16, bf16_to_u16

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H, D = 17, 128
SCALE = 1.0 / np.sqrt(128.0)
STATUS_DECODE_BOUND = 0x200  # decode.cu: a kv_len above max_kv_len was clamped


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _batch(lens, seed, heads):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows = max(lens) + 3

    def rnd(*shape):
        return torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)

    B = len(lens)
    q, kn, vn = rnd(B, heads, D), rnd(B, heads, D), rnd(B, heads, D)
    kcs = [rnd(rows, heads, D) for _ in lens]
    vcs = [rnd(rows, heads, D) for _ in lens]
    return q, kn, vn, kcs, vcs


def _ptr_table(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")


def _regular(lib, q, kn, vn, kcs, vcs, lens, mx, heads):
    """nc_decode_attention with a caller workspace, on its own copy of the caches."""
    B = len(lens)
    k_ref = [k.clone() for k in kcs]
    v_ref = [v.clone() for v in vcs]
    lt = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = torch.zeros(lib.nc_decode_workspace_bytes(B, mx, heads, 0), dtype=torch.uint8,
                     device="cuda")
    out = torch.empty((B, heads * D), dtype=torch.bfloat16, device="cuda")
    assert lib.nc_decode_attention(_p(out), _p(q), _p(kn), _p(vn), _p(_ptr_table(k_ref)),
                                   _p(_ptr_table(v_ref)), _p(lt), B, heads, SCALE, mx, 0, _p(ws),
                                   ws.numel(), _stream()) == 0
    torch.cuda.synchronize()
    return out, k_ref, v_ref


def _noalloc_twice(lib, q, kn, vn, kcs, vcs, lens, mx, heads, want, what):
    """Two allocation-free calls in a row on the same caches; each must give `want` (the
    second call re-appends the same new rows, so it sees the same caches)."""
    B = len(lens)
    kt, vt = _ptr_table(kcs), _ptr_table(vcs)
    lt = torch.tensor(lens, dtype=torch.int32, device="cuda")
    for call in range(2):
        out = torch.full((B, heads * D), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = lib.nc_decode_attention_noalloc(_p(out), _p(q), _p(kn), _p(vn), _p(kt), _p(vt),
                                             _p(lt), B, heads, SCALE, mx, _stream())
        assert st == 0, lib.nc_status_string(st)
        torch.cuda.synchronize()
        assert_close_bf16(bf16_to_u16(out), want, what=f"{what} call {call}")


@pytest.mark.parametrize("lens,heads", [
    ([1, 17, 300, 2048], H),      # per-head layout, several splits
    ([5] * 3 + [4000], H),        # streaming layout
    ([129] * 64, H),              # streaming layout, many sequences
    ([1], H),                     # one key: one split, no partials
    ([20000], H),                 # one long sequence: many splits on the streaming layout
    ([2048] * 256, H),            # largest batch: the split length grows to fit the array
])
def test_noalloc_matches_workspace_entry_point(lens, heads):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc

    lib = nc.load()
    nc.init_rope_tables()
    mx = max(lens)
    q, kn, vn, kcs, vcs = _batch(lens, seed=len(lens) + mx, heads=heads)
    out_ref, k_ref, v_ref = _regular(lib, q, kn, vn, kcs, vcs, lens, mx, heads)
    _noalloc_twice(lib, q, kn, vn, kcs, vcs, lens, mx, heads, bf16_to_u16(out_ref),
                   what=f"noalloc vs workspace lens={lens[:4]}")
    # the appended key/value rows agree with the regular entry point's
    for b in range(len(lens)):
        assert torch.equal(kcs[b], k_ref[b]) and torch.equal(vcs[b], v_ref[b])
    assert nc.device_status(reset=True) == 0


@pytest.mark.parametrize("lens", [[1, 17, 300, 2048], [7, 640, 1500, 33, 2047] * 3])
def test_noalloc_matches_oracle(lens):
    """Against the CPU oracle directly (RoPE + QK-norm of q and of the new key, append, split
    attention), on RMS-normalised caches as a model produces them."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc

    lib = nc.load()
    nc.init_rope_tables()
    mx, B = max(lens), len(lens)
    q, kn, vn, kcs, vcs = _batch(lens, seed=31 + mx, heads=H)
    for kc in kcs:
        nc.apply_rope_rmsnorm(kc, kc.shape[0], H, 0)
    torch.cuda.synchronize()
    hk = [bf16_to_u16(k) for k in kcs]
    hv = [bf16_to_u16(v) for v in vcs]
    want, _, _ = oracle.decode_step(bf16_to_u16(q), bf16_to_u16(kn), bf16_to_u16(vn), hk, hv,
                                    lens, H, SCALE)
    _noalloc_twice(lib, q, kn, vn, kcs, vcs, lens, mx, H, want.reshape(B, H * D),
                   what=f"noalloc vs oracle lens={lens[:4]}")
    assert nc.device_status(reset=True) == 0


def test_noalloc_clamps_length_above_bound():
    """A kv_len above max_kv_len is clamped to max_kv_len and flagged in the status word, as by
    the regular entry point."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc

    lib = nc.load()
    nc.init_rope_tables()
    lens, mx = [100, 700, 300], 500   # 700 > max_kv_len
    q, kn, vn, kcs, vcs = _batch(lens, seed=77, heads=H)
    nc.device_status(reset=True)
    out_ref, _, _ = _regular(lib, q, kn, vn, kcs, vcs, lens, mx, H)
    assert nc.device_status(reset=True) & STATUS_DECODE_BOUND
    _noalloc_twice(lib, q, kn, vn, kcs, vcs, lens, mx, H, bf16_to_u16(out_ref),
                   what="noalloc clamped")
    assert nc.device_status(reset=True) & STATUS_DECODE_BOUND


def test_noalloc_rejects_beyond_its_limits():
    import nanochat_inferonly_lightning_b200 as nc

    lib = nc.load()
    P = ctypes.c_void_p
    # batch above 256 and kv_len above the RoPE table are refused before any device work
    assert lib.nc_decode_attention_noalloc(P(256), P(256), None, None, P(256), P(256), P(256),
                                           257, H, SCALE, 128, None) == 7
    assert lib.nc_decode_attention_noalloc(P(256), P(256), None, None, P(256), P(256), P(256),
                                           4, H, SCALE, 20481, None) == 7

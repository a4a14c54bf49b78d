"""GPU parity of the CUDA path (called through the C ABI) against the CPU oracle and against
the reference's own kernels rebuilt for sm_100a.

Tolerance for attention outputs (bf16): max-abs 2e-2 and mean-abs 2e-3; NaN positions equal.
RoPE alone is bit-exact against the oracle (same fp32 table, same fused multiply-adds); RoPE +
QK-norm may differ by one bf16 ulp where the GPU's rsqrt and the oracle's 1/sqrt round apart.
"""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import assert_close_bf16, bf16_to_u16, u16_to_bf16, ulp_diff_bf16

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

H = 17
D = 128
SCALE = 1.0 / np.sqrt(128.0)


@pytest.fixture(scope="module")
def nc():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as m

    m.init_rope_tables()
    yield m
    torch.cuda.synchronize()
    assert m.device_status(reset=True) == 0, "a kernel's bounded wait gave up"


@pytest.fixture(scope="module")
def ref():
    lib = oracle.reference_kernels()
    if lib is None:
        pytest.skip("reference kernels not built (oracle/_ref)")
    assert lib.ref_init_rope_tables() == 0
    return lib


def randn_u16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    t = (torch.randn(shape, generator=g, dtype=torch.float32) * scale).to(torch.bfloat16)
    return bf16_to_u16(t)


def normed(x_u16, start_pos=0):
    """RoPE + QK-norm by the oracle (rows are positions start_pos..)."""
    return oracle.apply_rope_rmsnorm(x_u16, x_u16.shape[0], x_u16.shape[1], start_pos)


def dev(a_u16):
    return u16_to_bf16(a_u16, "cuda")


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def guarded(n_elems, guard=4096):
    """A device buffer with poisoned guard regions before and after the payload."""
    buf = torch.full((n_elems + 2 * guard,), float("nan"), dtype=torch.bfloat16, device="cuda")
    buf.view(torch.int16).fill_(0x5A5A)
    return buf, buf[guard:guard + n_elems]


def guards_intact(buf, guard=4096):
    v = buf.view(torch.int16)
    return bool((v[:guard] == 0x5A5A).all()) and bool((v[-guard:] == 0x5A5A).all())


# ----------------------------------------------------------------------------- RoPE tables
def test_reference_rope_table_matches_oracle(ref):
    """Pins the oracle's table to the reference's own init_rope_tables (bit-exact)."""
    n = 20480
    c = np.zeros((n, 64), np.float32)
    s = np.zeros((n, 64), np.float32)
    assert ref.ref_get_rope_tables(c.ctypes.data_as(ctypes.c_void_p),
                                   s.ctypes.data_as(ctypes.c_void_p), n) == 0
    oc, os_ = oracle.rope_tables()
    assert np.array_equal(c.view(np.uint32), oc.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))


# ----------------------------------------------------------------------------- RoPE
@pytest.mark.parametrize("seq_len,start_pos", [(1, 0), (3, 511), (64, 1000), (129, 20480 - 129)])
def test_apply_rope_bit_exact(nc, ref, seq_len, start_pos):
    x = randn_u16((seq_len, H, D), 10 + seq_len)
    want = oracle.apply_rope(x, seq_len, H, start_pos)
    t = dev(x)
    nc.apply_rope(t, seq_len, H, start_pos)
    got = bf16_to_u16(t)
    assert np.array_equal(got, want)
    # the reference kernel agrees with the oracle to one bf16 ulp
    r = dev(x)
    assert ref.ref_apply_rope(ctypes.c_void_p(r.data_ptr()), seq_len, H, start_pos, stream_ptr()) == 0
    torch.cuda.synchronize()
    assert ulp_diff_bf16(bf16_to_u16(r), want).max() <= 1


@pytest.mark.parametrize("seq_len,start_pos", [(1, 511), (7, 0), (128, 1536), (300, 17)])
def test_apply_rope_rmsnorm(nc, ref, seq_len, start_pos):
    x = randn_u16((seq_len, H, D), 20 + seq_len)
    want = oracle.apply_rope_rmsnorm(x, seq_len, H, start_pos)
    t = dev(x)
    nc.apply_rope_rmsnorm(t, seq_len, H, start_pos)
    got = bf16_to_u16(t)
    d = ulp_diff_bf16(got, want)
    assert d.max() <= 1 and (d == 0).mean() >= 0.99
    r = dev(x)
    assert ref.ref_apply_rope_rmsnorm(ctypes.c_void_p(r.data_ptr()), seq_len, H, start_pos,
                                      stream_ptr()) == 0
    torch.cuda.synchronize()
    dr = ulp_diff_bf16(bf16_to_u16(r), want)
    assert dr.max() <= 1 and (dr == 0).mean() >= 0.99
    # mine against the reference kernel directly
    assert ulp_diff_bf16(got, bf16_to_u16(r)).max() <= 1


@pytest.mark.parametrize("seq_len,start_pos", [(1, 0), (5, 100), (512, 1536)])
def test_rope_qknorm_append(nc, seq_len, start_pos):
    rows = start_pos + seq_len + 3
    q = randn_u16((seq_len, H, D), 30)
    k = randn_u16((seq_len, H, D), 31)
    v = randn_u16((seq_len, H, D), 32)
    kc0 = randn_u16((rows, H, D), 33)
    vc0 = randn_u16((rows, H, D), 34)
    wq, wkc, wvc = oracle.rope_qknorm_append(q, k, v, kc0, vc0, seq_len, H, start_pos)
    tq, tk, tv, tkc, tvc = dev(q), dev(k), dev(v), dev(kc0), dev(vc0)
    nc.rope_qknorm_append(tq, tk, tv, tkc, tvc, seq_len, H, start_pos)
    assert ulp_diff_bf16(bf16_to_u16(tq), wq).max() <= 1
    assert ulp_diff_bf16(bf16_to_u16(tkc), wkc).max() <= 1
    assert np.array_equal(bf16_to_u16(tvc), wvc)
    # inputs k, v untouched; rows outside the append window untouched
    assert np.array_equal(bf16_to_u16(tk), k) and np.array_equal(bf16_to_u16(tv), v)
    assert np.array_equal(bf16_to_u16(tkc)[:start_pos], kc0[:start_pos])
    assert np.array_equal(bf16_to_u16(tkc)[start_pos + seq_len:], kc0[start_pos + seq_len:])


@pytest.mark.parametrize("batch,seq_len,start_pos", [(1, 3, 0), (3, 37, 0), (8, 64, 100)])
def test_rope_qknorm_append_batched(nc, batch, seq_len, start_pos):
    """One launch over `batch` sequences equals `batch` single-sequence appends (the oracle per
    sequence): each chunk lands in its own cache slot, rows outside the window untouched."""
    slot_rows = start_pos + seq_len + 5
    q = randn_u16((batch * seq_len, H, D), 40)
    k = randn_u16((batch * seq_len, H, D), 41)
    v = randn_u16((batch * seq_len, H, D), 42)
    kc0 = randn_u16((batch, slot_rows, H, D), 43)
    vc0 = randn_u16((batch, slot_rows, H, D), 44)
    tq, tk, tv, tkc, tvc = dev(q), dev(k), dev(v), dev(kc0), dev(vc0)
    nc.rope_qknorm_append_batched(tq, tk, tv, tkc, tvc, slot_rows * H * D, batch, seq_len, H,
                                  start_pos)
    gq, gkc, gvc = bf16_to_u16(tq), bf16_to_u16(tkc), bf16_to_u16(tvc)
    for b in range(batch):
        r = slice(b * seq_len, (b + 1) * seq_len)
        wq, wkc, wvc = oracle.rope_qknorm_append(q[r], k[r], v[r], kc0[b], vc0[b], seq_len, H,
                                                 start_pos)
        assert ulp_diff_bf16(gq[r], wq).max() <= 1
        assert ulp_diff_bf16(gkc[b], wkc).max() <= 1
        assert np.array_equal(gvc[b], wvc)
        assert np.array_equal(gkc[b][:start_pos], kc0[b][:start_pos])
        assert np.array_equal(gkc[b][start_pos + seq_len:], kc0[b][start_pos + seq_len:])


def test_rope_qknorm_append_batched_rejects_short_stride(nc):
    t = dev(randn_u16((2 * 4, H, D), 45))
    c = dev(randn_u16((2, 4, H, D), 46))
    with pytest.raises(RuntimeError):
        nc.rope_qknorm_append_batched(t, t.clone(), t.clone(), c, c.clone(), 3 * H * D, 2, 4, H, 0)


# ----------------------------------------------------------------------------- prefill
PREFILL_CASES = [
    # (seq_q, kv_len, kv_offset)
    (2, 2, 0),
    (7, 7, 0),
    (63, 63, 0),
    (128, 128, 0),
    (129, 129, 0),
    (200, 1736, 1536),
    (128, 2048, 1920),
    (512, 2048, 1536),
    (1, 1, 0),
    (16, 100, 200),      # kv_offset beyond kv_len: every row sees all 100 keys
    (300, 300, 0),
]


def _attention_case(nc, ref, seq_q, kv_len, off, seed, qk_scale=1.0, normalise=True,
                    scale=SCALE):
    q = randn_u16((seq_q, H, D), seed, qk_scale)
    k = randn_u16((kv_len, H, D), seed + 1, qk_scale)
    v = randn_u16((kv_len, H, D), seed + 2)
    if normalise:
        q = normed(q, max(off, 0))
        k = normed(k, 0)
    want = oracle.flash_attention(q, k, v, seq_q, kv_len, H, scale, off)
    buf, out = guarded(seq_q * H * D)
    nc.flash_attention(out, dev(q), dev(k), dev(v), seq_q, kv_len, H, scale, off)
    torch.cuda.synchronize()
    assert guards_intact(buf), "kernel wrote outside its output"
    got = bf16_to_u16(out).reshape(seq_q, H * D)
    assert_close_bf16(got, want, what=f"mine seq_q={seq_q} kv={kv_len} off={off}")
    if ref is not None and seq_q * kv_len <= 600_000:
        r = torch.empty((seq_q, H * D), dtype=torch.bfloat16, device="cuda")
        tq, tk, tv = dev(q), dev(k), dev(v)
        assert ref.ref_flash_attention(ctypes.c_void_p(r.data_ptr()), ctypes.c_void_p(tq.data_ptr()),
                                       ctypes.c_void_p(tk.data_ptr()), ctypes.c_void_p(tv.data_ptr()),
                                       seq_q, kv_len, H, float(scale), off, stream_ptr()) == 0
        torch.cuda.synchronize()
        rr = bf16_to_u16(r)
        assert_close_bf16(rr, want, what="reference kernel vs oracle")
        assert_close_bf16(got, rr, what="mine vs reference kernel")
    return got, want


@pytest.mark.parametrize("seq_q,kv_len,off", PREFILL_CASES)
def test_flash_attention_prefill(nc, ref, seq_q, kv_len, off):
    _attention_case(nc, ref, seq_q, kv_len, off, seed=1000 + seq_q + kv_len)


def test_flash_attention_prefill_full_2048(nc, ref):
    """cfg2 shape (2048 positions, causal, empty cache): against the oracle."""
    _attention_case(nc, None, 2048, 2048, 0, seed=7)


def test_flash_attention_prefill_wide_scores(nc):
    """Unnormalised, scaled inputs (scores spread over tens of units) exercise the lazy
    rescale of O and of the row sum."""
    _attention_case(nc, None, 256, 640, 384, seed=99, qk_scale=3.0, normalise=False)


def test_flash_attention_prefill_scores_far_below_bound(nc):
    """A large softmax scale on RMS-normalised inputs: the kernel's starting reference max (the
    bound 128 * scale * log2(e)) sits far above every block max, so a tile's first block has
    a row sum below 2^-64 and is redone with its own max."""
    _attention_case(nc, None, 256, 640, 384, seed=123, scale=0.5)


def test_flash_attention_prefill_no_visible_key(nc):
    """kv_offset < 0: leading rows see no key and become NaN, like the reference's 0/0."""
    _attention_case(nc, None, 150, 150, -20, seed=5)


def test_flash_attention_zero_kv(nc):
    out = torch.zeros((3, H * D), dtype=torch.bfloat16, device="cuda")
    z = torch.zeros((1, H, D), dtype=torch.bfloat16, device="cuda")
    nc.flash_attention(out, torch.zeros((3, H, D), dtype=torch.bfloat16, device="cuda"), z, z,
                       3, 0, H, SCALE, 0)
    torch.cuda.synchronize()
    assert torch.isnan(out.float()).all()


# ----------------------------------------------------------------------------- decode
@pytest.mark.parametrize("kv_len", [1, 2, 15, 16, 17, 63, 64, 129, 511, 512, 1536 + 512, 4097])
def test_flash_attention_decode(nc, ref, kv_len):
    """seq_q == 1 through the reference entry point (split-KV decode kernel)."""
    _attention_case(nc, ref, 1, kv_len, kv_len - 1, seed=2000 + kv_len)


def test_flash_attention_decode_offset_limits_keys(nc):
    """Single query with kv_offset < kv_len - 1: only keys <= kv_offset are visible."""
    _attention_case(nc, None, 1, 700, 300, seed=77)


def _decode_batch(nc, lens, split_len, seed, fused=True, rows_extra=5):
    B = len(lens)
    max_len = max(lens)
    rows = max_len + rows_extra
    q = randn_u16((B, H, D), seed)
    kn = randn_u16((B, H, D), seed + 1)
    vn = randn_u16((B, H, D), seed + 2)
    kcs, vcs = [], []
    for b, L in enumerate(lens):
        kc = normed(randn_u16((rows, H, D), seed + 10 + 2 * b), 0)
        vc = randn_u16((rows, H, D), seed + 11 + 2 * b)
        kcs.append(kc)
        vcs.append(vc)
    if fused:
        want, wkc, wvc = oracle.decode_step(q, kn, vn, kcs, vcs, lens, H, SCALE)
    else:
        qn = np.stack([normed(q[b:b + 1], lens[b] - 1)[0] for b in range(B)])
        want, wkc, wvc = oracle.decode_step(qn, None, None, kcs, vcs, lens, H, SCALE)
        q = qn
    tk = [dev(k) for k in kcs]
    tv = [dev(v) for v in vcs]
    kp = torch.tensor([t.data_ptr() for t in tk], dtype=torch.int64, device="cuda")
    vp = torch.tensor([t.data_ptr() for t in tv], dtype=torch.int64, device="cuda")
    lt = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = torch.zeros(nc.decode_workspace_bytes(B, max_len, H, split_len), dtype=torch.uint8,
                     device="cuda")
    buf, out = guarded(B * H * D)
    for _ in range(2):  # second call checks the self-resetting split counters
        nc.decode_attention(out, dev(q), dev(kn) if fused else None, dev(vn) if fused else None,
                            kp, vp, lt, H, SCALE, max_len, ws, split_len=split_len)
        torch.cuda.synchronize()
        got = bf16_to_u16(out).reshape(B, H * D)
        assert_close_bf16(got, want, what=f"decode lens={lens} split={split_len}")
    assert guards_intact(buf)
    for b in range(B):
        gk, gv = bf16_to_u16(tk[b]), bf16_to_u16(tv[b])
        assert ulp_diff_bf16(gk, wkc[b]).max() <= 1, f"K cache of sequence {b}"
        assert np.array_equal(gv, wvc[b]), f"V cache of sequence {b}"


@pytest.mark.parametrize("split_len", [0, 16, 32, 128])
def test_decode_batched_fused(nc, split_len):
    _decode_batch(nc, [1, 2, 17, 100, 513, 1200], split_len, seed=300)


def test_decode_batched_unfused(nc):
    _decode_batch(nc, [3, 64, 65, 700], 0, seed=400, fused=False)


def test_decode_batched_head_layout_many_sequences(nc):
    """Up to 16 sequences and 16384 keys in all take the per-head layout: 12 ragged sequences,
    the longest with 21 splits (global combine) and the shortest with one."""
    _decode_batch(nc, [1, 40, 64, 65, 200, 333, 512, 700, 900, 1100, 1250, 1300], 0, seed=430)


def test_decode_batched_streaming_layout(nc):
    """More than 8 sequences: the streaming layout (all heads of a split per work item, CTAs
    taking items from a queue), with automatic splits."""
    _decode_batch(nc, [1, 5, 16, 33, 64, 128, 300, 511, 777, 1024, 1500, 2047], 0, seed=450)


@pytest.mark.parametrize("lens,page_rows,heads,split_len", [
    ([1, 2, 17, 100, 513, 1200], 64, H, 0),          # per-head layout
    ([300, 7, 64, 65], 16, H, 0),                     # per-head layout, small pages
    ([1, 5, 16, 33, 64, 128, 300, 511, 777, 1024, 1500, 2047], 48, H, 0),  # streaming
    ([40, 700, 1300], 128, H, 80),                    # streaming, explicit split
    ([3, 90, 250, 600, 1000, 11, 77, 500, 333], 16, 20, 80),  # streaming, 6-row stages
])
def test_decode_paged(nc, lens, page_rows, heads, split_len):
    """nc_decode_attention_paged: K/V rows live in shuffled pages of two pools; the new key and
    value are appended through the page table.  Output against the oracle on the equivalent
    contiguous caches, appended rows in the right pages, spare pages untouched."""
    B, max_len = len(lens), max(lens)
    pps = -(-max_len // page_rows)
    num_pages = B * pps + 3
    rng = np.random.default_rng(700 + page_rows)
    perm = rng.permutation(num_pages).astype(np.int32)
    table = perm[:B * pps].reshape(B, pps)
    q = randn_u16((B, heads, D), 710)
    kn = randn_u16((B, heads, D), 711)
    vn = randn_u16((B, heads, D), 712)
    kcs = [normed(randn_u16((pps * page_rows, heads, D), 720 + b), 0) for b in range(B)]
    vcs = [randn_u16((pps * page_rows, heads, D), 760 + b) for b in range(B)]
    want, wkc, wvc = oracle.decode_step(q, kn, vn, kcs, vcs, lens, heads, SCALE)
    kpool = np.zeros((num_pages, page_rows, heads, D), np.uint16)
    vpool = np.zeros_like(kpool)
    for b in range(B):
        for j in range(pps):
            kpool[table[b, j]] = kcs[b][j * page_rows:(j + 1) * page_rows]
            vpool[table[b, j]] = vcs[b][j * page_rows:(j + 1) * page_rows]
    tk, tv = dev(kpool), dev(vpool)
    pt = torch.tensor(table, dtype=torch.int32, device="cuda")
    lt = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = torch.zeros(nc.decode_workspace_bytes(B, max_len, heads, split_len), dtype=torch.uint8,
                     device="cuda")
    out = torch.empty((B, heads * D), dtype=torch.bfloat16, device="cuda")
    nc.decode_attention_paged(out, dev(q), dev(kn), dev(vn), tk, tv, pt, lt, heads, SCALE,
                              max_len, ws, split_len=split_len)
    torch.cuda.synchronize()
    assert_close_bf16(bf16_to_u16(out).reshape(B, heads * D), want, what=f"paged {lens}")
    gk, gv = bf16_to_u16(tk), bf16_to_u16(tv)
    for b, L in enumerate(lens):
        pg, row = table[b, (L - 1) // page_rows], (L - 1) % page_rows
        assert ulp_diff_bf16(gk[pg, row], wkc[b][L - 1]).max() <= 1, f"appended K, seq {b}"
        assert np.array_equal(gv[pg, row], wvc[b][L - 1]), f"appended V, seq {b}"
    spare = perm[B * pps:]
    assert not gk[spare].any() and not gv[spare].any()
    assert nc.device_status(reset=True) == 0


def test_decode_paged_bad_page_id_is_flagged(nc):
    """A page id outside the pool is not dereferenced: the call completes, the status word gets
    the bounds bit, and the pool is not written."""
    B, page_rows, pps, num_pages = 2, 16, 4, 8
    lens = [40, 50]
    table = np.array([[0, 1, 2, 3], [4, 5, 99, 7]], np.int32)  # row 32.. of seq 1: bad page
    kpool = torch.zeros((num_pages, page_rows, H, D), dtype=torch.bfloat16, device="cuda")
    vpool = torch.zeros_like(kpool)
    q = dev(randn_u16((B, H, D), 790))
    out = torch.empty((B, H * D), dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(nc.decode_workspace_bytes(B, 64, H), dtype=torch.uint8, device="cuda")
    nc.device_status(reset=True)
    nc.decode_attention_paged(out, q, q, q, kpool, vpool,
                              torch.tensor(table, device="cuda"),
                              torch.tensor(lens, dtype=torch.int32, device="cuda"), H, SCALE,
                              64, ws)
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) & 0x400
    # only the two appended rows were written: row 39 of seq 0 (page 2), row 49 of seq 1 (page 7)
    for pg in (0, 1, 3, 4, 5, 6):
        assert int(kpool[pg].count_nonzero()) == 0 and int(vpool[pg].count_nonzero()) == 0
    assert int(kpool[2, 39 % 16].count_nonzero()) > 0 and int(kpool[7, 49 % 16].count_nonzero()) > 0


@pytest.mark.parametrize("lens", [
    [257, 300, 333, 401, 450, 479, 505, 520],                       # the engine's 8 sequences
    [64, 129, 300, 450, 520, 700, 800, 950, 1000, 1100, 1200, 1300],  # 12: up to 21 splits
])
def test_decode_overlap_after_qkv_gemm(nc, lens):
    """nc_decode_attention_overlap right after the fused Q/K/V GEMM that produces its q, k_new
    and v_new (the engine's order): the attention CTAs load cache rows while the GEMM runs and
    wait for it before reading q/k/v.  Same bits as the plain call made after a synchronize, and
    the oracle's result for the GEMM's q/k/v.  Both cases take the per-head layout (up to 16
    sequences and 16384 keys); the second combines more than 8 splits per head."""
    B, max_len = len(lens), max(lens)
    g = torch.Generator(device="cuda").manual_seed(610)
    x = torch.randn((B, H * D), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((3 * H * D, H * D), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    kcs = [normed(randn_u16((max_len, H, D), 620 + b), 0) for b in range(B)]
    vcs = [randn_u16((max_len, H, D), 640 + b) for b in range(B)]
    lt = torch.tensor(lens, dtype=torch.int32, device="cuda")
    results = []
    for overlap in (True, False):
        tk, tv = [dev(k) for k in kcs], [dev(v) for v in vcs]
        kp = torch.tensor([t.data_ptr() for t in tk], dtype=torch.int64, device="cuda")
        vp = torch.tensor([t.data_ptr() for t in tv], dtype=torch.int64, device="cuda")
        ws = torch.zeros(nc.decode_workspace_bytes(B, max_len, H), dtype=torch.uint8,
                         device="cuda")
        qkv = torch.empty((3, B, H * D), dtype=torch.bfloat16, device="cuda")
        out = torch.empty((B, H * D), dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        nc.gemm.gemm_skinny(qkv, x, w, flags=nc.gemm.NORM_INPUT, seg_cols=H * D)
        if not overlap:
            torch.cuda.synchronize()
        nc.decode_attention(out, qkv[0], qkv[1], qkv[2], kp, vp, lt, H, SCALE, max_len, ws,
                            overlap=overlap)
        torch.cuda.synchronize()
        results.append((bf16_to_u16(out), [bf16_to_u16(t) for t in tk],
                        [bf16_to_u16(t) for t in tv], bf16_to_u16(qkv)))
    (o1, k1, v1, qkv1), (o2, k2, v2, qkv2) = results
    assert np.array_equal(qkv1, qkv2) and np.array_equal(o1, o2)
    assert all(np.array_equal(a, b) for a, b in zip(k1, k2))
    assert all(np.array_equal(a, b) for a, b in zip(v1, v2))
    qkv1 = qkv1.reshape(3, B, H, D)
    want, _, _ = oracle.decode_step(qkv1[0], qkv1[1], qkv1[2], kcs, vcs, lens, H, SCALE)
    assert_close_bf16(o1.reshape(B, H * D), want, what="overlapped decode")


def test_decode_cfg3_lengths_subset(nc):
    """First 8 sequences of cfg3's kv_len draw (torch seed 2)."""
    from nanochat_inferonly_lightning_b200 import workloads

    _decode_batch(nc, workloads.cfg3_kv_lens()[:8], 0, seed=500)


# ----------------------------------------------------------------------------- batched prefill
@pytest.mark.parametrize("B,chunk,off,rows", [(2, 37, 100, 200), (3, 128, 1536, 2048),
                                              (2, 512, 0, 600)])
def test_prefill_batched(nc, B, chunk, off, rows):
    q = np.stack([normed(randn_u16((chunk, H, D), 600 + b), off) for b in range(B)])
    kslab = np.stack([normed(randn_u16((rows, H, D), 700 + b), 0) for b in range(B)])
    vslab = np.stack([randn_u16((rows, H, D), 800 + b) for b in range(B)])
    want = np.stack([oracle.flash_attention(q[b], kslab[b], vslab[b], chunk, off + chunk, H,
                                            SCALE, off) for b in range(B)])
    out = torch.empty((B, chunk, H * D), dtype=torch.bfloat16, device="cuda")
    offs = torch.full((B,), off, dtype=torch.int32, device="cuda")
    nc.prefill_attention_batched(out, dev(q), dev(kslab), dev(vslab), rows * H * D, rows, offs,
                                 chunk, H, SCALE)
    torch.cuda.synchronize()
    assert_close_bf16(bf16_to_u16(out), want, what="batched prefill")


@pytest.mark.parametrize("offs,chunk,page_rows", [([0, 200, 700], 300, 128),
                                                   ([1536, 0], 512, 256)])
def test_prefill_paged(nc, offs, chunk, page_rows):
    """Chunked prefill over a paged cache: nc_rope_qknorm_append_paged writes each sequence's
    chunk into its (shuffled) pages, crossing page edges; nc_prefill_attention_paged then reads
    the keys through the page table.  Against the oracle on the equivalent contiguous caches."""
    B = len(offs)
    pps = -(-max(o + chunk for o in offs) // page_rows)
    num_pages = B * pps + 2
    rng = np.random.default_rng(800 + page_rows)
    perm = rng.permutation(num_pages).astype(np.int32)
    table = perm[:B * pps].reshape(B, pps)
    kpool = np.zeros((num_pages, page_rows, H, D), np.uint16)
    vpool = np.zeros_like(kpool)
    qs, ks, vs, wants, wks, wvs, wqs = [], [], [], [], [], [], []
    for b, off in enumerate(offs):
        kc = np.zeros((pps * page_rows, H, D), np.uint16)
        vc = np.zeros_like(kc)
        if off:
            kc[:off] = normed(randn_u16((off, H, D), 810 + b), 0)
            vc[:off] = randn_u16((off, H, D), 820 + b)
        q, k, v = (randn_u16((chunk, H, D), 830 + 3 * b + i) for i in range(3))
        wq, wkc, wvc = oracle.rope_qknorm_append(q, k, v, kc, vc, chunk, H, off)
        wants.append(oracle.flash_attention(wq, wkc, wvc, chunk, off + chunk, H, SCALE, off))
        for j in range(pps):
            kpool[table[b, j]] = kc[j * page_rows:(j + 1) * page_rows]
            vpool[table[b, j]] = vc[j * page_rows:(j + 1) * page_rows]
        qs.append(q), ks.append(k), vs.append(v), wks.append(wkc), wvs.append(wvc), wqs.append(wq)
    tk, tv = dev(kpool), dev(vpool)
    tq = dev(np.stack(qs))
    for b, off in enumerate(offs):
        nc.rope_qknorm_append_paged(tq[b], dev(ks[b]), dev(vs[b]), tk, tv, list(table[b]), chunk,
                                    H, off)
    out = torch.empty((B, chunk, H * D), dtype=torch.bfloat16, device="cuda")
    nc.prefill_attention_paged(out, tq, tk, tv, torch.tensor(table, device="cuda"),
                               torch.tensor(offs, dtype=torch.int32, device="cuda"), chunk, H,
                               SCALE)
    torch.cuda.synchronize()
    gk, gv = bf16_to_u16(tk), bf16_to_u16(tv)
    for b, off in enumerate(offs):
        assert ulp_diff_bf16(bf16_to_u16(tq[b]), wqs[b]).max() <= 1
        rows = np.arange(off, off + chunk)
        got_k = gk[table[b, rows // page_rows], rows % page_rows]
        got_v = gv[table[b, rows // page_rows], rows % page_rows]
        assert ulp_diff_bf16(got_k, wks[b][off:off + chunk]).max() <= 1
        assert np.array_equal(got_v, wvs[b][off:off + chunk])
        assert_close_bf16(bf16_to_u16(out[b]), wants[b], what=f"paged prefill seq {b}")
    assert nc.device_status(reset=True) == 0


@pytest.mark.parametrize("B,chunk,start,page_rows", [(3, 200, 100, 128), (8, 64, 0, 16)])
def test_rope_qknorm_append_paged_batched(nc, B, chunk, start, page_rows):
    """One launch for every sequence of a device page table (shuffled pages, chunks crossing
    page edges) equals the oracle's append per sequence; the row of a sequence whose page id is
    out of range is skipped and reported in the status word."""
    pps = -(-(start + chunk) // page_rows)
    num_pages = B * pps + 3
    rng = np.random.default_rng(900 + page_rows)
    table = rng.permutation(num_pages).astype(np.int32)[:B * pps].reshape(B, pps)
    kpool0 = randn_u16((num_pages, page_rows, H, D), 901)
    vpool0 = randn_u16((num_pages, page_rows, H, D), 902)
    q = randn_u16((B * chunk, H, D), 903)
    k = randn_u16((B * chunk, H, D), 904)
    v = randn_u16((B * chunk, H, D), 905)
    tk, tv, tq = dev(kpool0), dev(vpool0), dev(q)
    nc.rope_qknorm_append_paged_batched(tq, dev(k), dev(v), tk, tv,
                                        torch.tensor(table, device="cuda"), chunk, H, start)
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) == 0
    gq, gk, gv = bf16_to_u16(tq), bf16_to_u16(tk), bf16_to_u16(tv)
    rows = np.arange(start, start + chunk)
    touched = np.zeros((num_pages, page_rows), bool)
    for b in range(B):
        r = slice(b * chunk, (b + 1) * chunk)
        kc = np.zeros((start + chunk, H, D), np.uint16)
        vc = np.zeros_like(kc)
        wq, wkc, wvc = oracle.rope_qknorm_append(q[r], k[r], v[r], kc, vc, chunk, H, start)
        assert ulp_diff_bf16(gq[r], wq).max() <= 1
        pg, pr = table[b, rows // page_rows], rows % page_rows
        assert ulp_diff_bf16(gk[pg, pr], wkc[start:]).max() <= 1
        assert np.array_equal(gv[pg, pr], wvc[start:])
        touched[pg, pr] = True
    assert np.array_equal(gk[~touched], kpool0[~touched])
    assert np.array_equal(gv[~touched], vpool0[~touched])

    # a page id outside [0, num_pages): that sequence's rows on the page are not written
    bad = table.copy()
    bad[0, -1] = num_pages
    tk2, tv2 = dev(kpool0), dev(vpool0)
    nc.rope_qknorm_append_paged_batched(dev(q), dev(k), dev(v), tk2, tv2,
                                        torch.tensor(bad, device="cuda"), chunk, H, start)
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) & 0x400
    g2 = bf16_to_u16(tk2)
    in_bad = rows // page_rows == pps - 1
    assert np.array_equal(g2[table[0, -1]], kpool0[table[0, -1]])
    assert np.array_equal(g2[bad[0, rows[~in_bad] // page_rows], rows[~in_bad] % page_rows],
                          gk[bad[0, rows[~in_bad] // page_rows], rows[~in_bad] % page_rows])


# ----------------------------------------------------------------------------- KV cache object
def test_kv_cache_prefill_then_decode(nc):
    """Prefill a prompt through the cache object, then decode steps for two sequences; the
    oracle replays the same sequence of appends."""
    n_seqs, max_len, prompt = 2, 300, 40
    cache = nc.KVCache(n_layers=2, n_seqs=n_seqs, max_len=max_len, heads=H)
    layer = 1
    okc = [np.zeros((max_len, H, D), np.uint16) for _ in range(n_seqs)]
    ovc = [np.zeros((max_len, H, D), np.uint16) for _ in range(n_seqs)]
    for s in range(n_seqs):
        q = randn_u16((prompt, H, D), 900 + s)
        k = randn_u16((prompt, H, D), 910 + s)
        v = randn_u16((prompt, H, D), 920 + s)
        wq, okc[s], ovc[s] = oracle.rope_qknorm_append(q, k, v, okc[s], ovc[s], prompt, H, 0)
        want = oracle.flash_attention(wq, okc[s], ovc[s], prompt, prompt, H, SCALE, 0)
        out = torch.empty((prompt, H * D), dtype=torch.bfloat16, device="cuda")
        cache.prefill(layer, s, out, dev(q), dev(k), dev(v), prompt, SCALE)
        torch.cuda.synchronize()
        assert_close_bf16(bf16_to_u16(out), want, what="cache prefill")
        assert cache.length(layer, s) == prompt
    for step in range(3):
        q = randn_u16((n_seqs, H, D), 950 + step)
        kn = randn_u16((n_seqs, H, D), 960 + step)
        vn = randn_u16((n_seqs, H, D), 970 + step)
        lens = [cache.length(layer, s) + 1 for s in range(n_seqs)]
        want, okc, ovc = oracle.decode_step(q, kn, vn, okc, ovc, lens, H, SCALE)
        out = torch.empty((n_seqs, H * D), dtype=torch.bfloat16, device="cuda")
        cache.decode(layer, out, dev(q), dev(kn), dev(vn), SCALE)
        torch.cuda.synchronize()
        assert_close_bf16(bf16_to_u16(out), want, what=f"cache decode step {step}")
    for s in range(n_seqs):
        assert cache.length(layer, s) == prompt + 3
        assert ulp_diff_bf16(bf16_to_u16(cache.view(layer, s, "k")), okc[s]).max() <= 1
        assert np.array_equal(bf16_to_u16(cache.view(layer, s, "v")), ovc[s])
    cache.clear()
    assert cache.length(layer, 0) == 0
    cache.close()


def test_device_status_clean(nc):
    torch.cuda.synchronize()
    assert nc.device_status() == 0

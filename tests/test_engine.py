"""Batched engine (nanochat_inferonly_lightning_b200/engine.py) on the full architecture:

* a decode step replayed from its CUDA graph gives exactly the tokens of the same step run
  eagerly (same kernels, same order);
* every decode step's logits match a recomputation of the whole sequence through the prefill
  path (tcgen05 prefill kernel over all positions, last row), within 0.25 in logit units, and
  greedy choices agree except where the recomputed logits of the two tokens are within 8 bf16
  ulps (the rounding floor of this random-weight network is ~6 ulps; see test_e2e_greedy.py).
"""
import math

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

B, PROMPT, STEPS, MAX_LEN = 4, 24, 8, 64


def bf16_ulp(x):
    e = math.floor(math.log2(max(abs(x), 2.0 ** -126)))
    return 2.0 ** (e - 7)


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import nanochat_inferonly_lightning_b200 as nc
    from nanochat_inferonly_lightning_b200 import engine as E

    w = E.Weights(seed=4)
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(2, E.VOCAB, (B, PROMPT), generator=g).cuda()
    yield nc, E, w, prompts
    torch.cuda.synchronize()
    assert nc.device_status(reset=True) == 0, "a kernel's bounded wait gave up"


def rmsnorm(x):
    """Parameter-free RMSNorm in fp32 (kernels/rmsnorm.cu: x * rsqrt(mean(x^2) + 1e-6))."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)


def logits_of(w, x, cap=15.0):
    """Final RMSNorm, LM head, tanh soft cap (src/model.cpp:147-155)."""
    lg = (rmsnorm(x) @ w.lm_head.t()).float()
    return (cap * torch.tanh(lg / cap)).to(torch.bfloat16)


def full_logits(E, w, seq_tokens):
    """Last-position logits of one sequence, recomputed independently of the engine: torch's
    RMSNorm and cuBLAS GEMMs around this library's prefill attention, over all positions."""
    import nanochat_inferonly_lightning_b200 as nc

    P = len(seq_tokens)
    kc = torch.zeros(P, E.N_HEAD, E.HEAD_DIM, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    x = rmsnorm(w.embed[torch.tensor(seq_tokens, device="cuda")])
    for l in w.layers:
        xn = rmsnorm(x)
        q, k, v = xn @ l["q"].t(), xn @ l["k"].t(), xn @ l["v"].t()
        a = torch.empty_like(q)
        nc.rope_qknorm_append(q, k, v, kc, vc, P, E.N_HEAD, 0)
        nc.flash_attention(a, q, kc, vc, P, P, E.N_HEAD, E.SCALE, 0)
        x = torch.addmm(x, a, l["o"].t())
        h = torch.relu(rmsnorm(x) @ l["up"].t()).square()
        x = torch.addmm(x, h, l["down"].t())
    return logits_of(w, x[-1:])[0].float()


def test_graph_replay_matches_eager(setup):
    nc, E, w, prompts = setup
    a = E.BatchedEngine(w, B, MAX_LEN)
    b = E.BatchedEngine(w, B, MAX_LEN)
    assert torch.equal(a.prefill(prompts), b.prefill(prompts))
    ta = [a.capture()]
    tb = [b.step().clone()]
    for _ in range(STEPS):
        ta.append(a.step().clone())
        tb.append(b.step().clone())
    assert torch.equal(torch.stack(ta), torch.stack(tb))
    assert int(a.kv_len[0]) == PROMPT + STEPS + 1


def test_decode_steps_match_prefill_recompute(setup):
    nc, E, w, prompts = setup
    eng = E.BatchedEngine(w, B, MAX_LEN)
    seqs = [list(map(int, p)) for p in prompts.cpu()]
    toks = eng.prefill(prompts)
    worst = 0.0
    for n in range(STEPS):
        for s in range(B):
            seqs[s].append(int(toks[s]))
        toks = eng.step().clone()
        for s in range(B):
            ref = full_logits(E, w, seqs[s])
            worst = max(worst, float((eng.logits[s].float() - ref).abs().max()))
            want, got = int(torch.argmax(ref)), int(toks[s])
            if got != want:
                gap = (float(ref[want]) - float(ref[got])) / bf16_ulp(float(ref[want]))
                assert gap <= 8.0, f"step {n} seq {s}: engine {got}, recompute {want} ({gap:.1f} ulps)"
                toks[s] = want  # follow the recompute so both stay on the same sequence
                eng.tok[s] = want
    assert worst < 0.25, worst


def test_sampled_decode_in_graph(setup):
    """Temperature / top-k / top-p sampling inside the captured step (device draws): every
    sampled token is among the top_k logits of its row, and two engines seeded alike sample the
    same tokens."""
    nc, E, w, prompts = setup
    runs = []
    for _ in range(2):
        eng = E.BatchedEngine(w, B, MAX_LEN, temperature=1.0, top_k=20, top_p=0.9, seed=123)
        eng.prefill(prompts)
        toks = [eng.capture()]
        for _ in range(4):
            t = eng.step().clone()
            kth = torch.topk(eng.logits.float(), 20, dim=-1).values[:, -1]
            chosen = eng.logits.float().gather(1, t.long()[:, None])[:, 0]
            assert bool((chosen >= kth).all())  # within the top 20 (ties at the edge allowed)
            toks.append(t)
        runs.append(torch.stack(toks))
    assert torch.equal(runs[0], runs[1])


def test_top_p_only_sampling_in_graph(setup):
    """top_k off and top_p 0.9 (Engine::top_p_filter over the whole vocabulary) inside the
    captured step: every sampled token lies in its row's nucleus (exact sums over the row sorted
    by descending probability, 1e-4 slack at the edge), and two engines seeded alike sample the
    same tokens."""
    nc, E, w, prompts = setup
    runs = []
    for _ in range(2):
        eng = E.BatchedEngine(w, B, MAX_LEN, temperature=0.8, top_k=0, top_p=0.9, seed=7)
        eng.prefill(prompts)
        toks = [eng.capture()]
        for _ in range(3):
            t = eng.step().clone()
            pr = torch.softmax(eng.logits.double() / 0.8, dim=-1)
            for s in range(B):
                srt, idx = torch.sort(pr[s], descending=True, stable=True)
                cs = torch.cumsum(srt, 0)
                pos = int((idx == int(t[s])).nonzero()[0, 0])
                assert pos == 0 or float(cs[pos - 1]) <= 0.9 + 1e-4, (s, pos)
            toks.append(t)
        runs.append(torch.stack(toks))
    assert torch.equal(runs[0], runs[1])


def test_continuous_batching(setup):
    """Sequences join and leave the running batch between graph replays (admit / retire)
    without re-capturing: a sequence admitted into slot 2 after three steps of slot 0 produces
    exactly the tokens it produces when it runs alone, slot 0 is unaffected by the newcomer,
    and a retired slot's length stops advancing."""
    nc, E, w, prompts = setup
    a = E.BatchedEngine(w, B, MAX_LEN)
    slot0 = [int(a.admit(0, prompts[0]))]
    slot0.append(int(a.capture()[0]))  # one eager step, then the capture
    for _ in range(2):
        slot0.append(int(a.step()[0]))
    slot2 = [int(a.admit(2, prompts[2]))]
    for _ in range(4):
        t = a.step().clone()
        slot0.append(int(t[0]))
        slot2.append(int(t[2]))
    a.retire(0)
    n0 = int(a.kv_len[0])
    a.step()
    assert int(a.kv_len[0]) == n0 and int(a.kv_len[2]) == PROMPT + 5

    def alone(slot, n_tokens):
        e = E.BatchedEngine(w, B, MAX_LEN)
        toks = [int(e.admit(slot, prompts[slot])), int(e.capture()[slot])]
        while len(toks) < n_tokens:
            toks.append(int(e.step()[slot]))
        return toks

    assert slot2 == alone(2, len(slot2))
    assert slot0 == alone(0, len(slot0))


def test_paged_engine_matches_contiguous(setup):
    """PagedEngine (pages of 128 rows from a shared pool, a host allocator, the library's paged
    prefill / append / decode) gives the contiguous engine's tokens and logits exactly: prompts
    of 120 tokens, then steps that cross into each sequence's second page.  A retired slot's
    pages go back to the pool and a sequence admitted there gets fresh ones."""
    nc, E, w, _ = setup
    g = torch.Generator().manual_seed(9)
    P, max_len, steps = 120, 256, 12
    prompts = torch.randint(2, E.VOCAB, (B, P), generator=g).cuda()
    ref = E.BatchedEngine(w, B, max_len)
    pg = E.PagedEngine(w, B, max_len, page_rows=128)
    assert torch.equal(ref.prefill(prompts), pg.prefill(prompts))
    assert pg.pages_in_use() == B
    assert torch.equal(ref.capture(), pg.capture())
    for _ in range(steps):
        assert torch.equal(ref.step(), pg.step())
        assert torch.equal(ref.logits, pg.logits)
    assert pg.pages_in_use() == 2 * B  # rows 0..132: two pages per sequence
    # retire slot 1 and admit a new sequence there in both engines
    ref.retire(1), pg.retire(1)
    assert pg.pages_in_use() == 2 * B - 2
    newp = torch.randint(2, E.VOCAB, (P,), generator=g).cuda()
    assert int(ref.admit(1, newp)) == int(pg.admit(1, newp))
    for _ in range(3):
        a, b = ref.step().clone(), pg.step().clone()
        for s in (0, 1, 2, 3):
            assert int(a[s]) == int(b[s]), s
    assert pg.pages_in_use() == 2 * (B - 1) + 1

"""Batched greedy generation on the reference model's architecture, with its attention path on
this library.

The forward pass follows the reference's Model (src/model.cpp:101-167): embedding, RMSNorm;
per layer RMSNorm -> Q/K/V projections -> RoPE + QK-norm -> KV append -> causal attention ->
output projection + residual, then RMSNorm -> MLP up -> ReLU^2 -> down + residual; final RMSNorm,
LM head, tanh soft cap 15.  Sampling is the reference's greedy rule (src/engine.cpp:88-95,
first maximum).  Weights use the reference's layout W[out, in] (src/model.h:30-47).

What runs where:
* the attention path (the part this library replaces) on this library: for a prompt pass over
  all slots, one nc_rope_qknorm_append_batched and one nc_prefill_attention_batched per layer
  (tcgen05 prefill; `admit` of one sequence uses the single-sequence calls); for each decode
  step, one nc_decode_attention over the whole batch (RoPE + QK-norm of q and k, append, and
  split-KV attention in one kernel), reading per-sequence lengths from a device array;
* the decode step's GEMMs on this library's skinny tcgen05 GEMM (gemm.py, nc_gemm_skinny): one
  pass over a fused [q; k; v] weight writing q, k and v separately, the output projection and
  MLP down projection with the residual added in place, the MLP up projection with ReLU^2, and
  the LM head with the tanh cap; the RMSNorm before the Q/K/V, MLP-up and LM-head GEMMs is a
  per-row scale applied inside them.  A decode layer is four GEMM launches and one attention
  launch; the step starts with one embedding-gather + RMSNorm launch and ends with an argmax
  launch on the device (gemm.py);
* the prompt pass (all sequences' B*P rows together; `admit` runs one sequence) on this library
  too: the embedding gather + RMSNorm kernel, the prompt-pass tcgen05 GEMM (nc_gemm) with the
  same fused steps as the decode step (RMSNorm row scale for Q/K/V and the MLP up projection,
  ReLU^2, the residual added in place), the attention's batched RoPE/QK-norm/append pass and
  batched tcgen05 prefill, and for the last position of each sequence the LM head on the skinny GEMM
  with the final RMSNorm and tanh cap fused, then the device argmax.

A decode step has static shapes and no host-side state, so it is captured once in a CUDA graph
and replayed; the device length array advances inside the graph.  The reference engine runs one
sequence at a time with host-side lengths (src/engine.cpp:37-62); here a batch of sequences
advances together.
"""
import math

import torch

from . import attn
from . import gemm as G

N_LAYER = 34
N_HEAD = 17
HEAD_DIM = 128
N_EMBD = N_HEAD * HEAD_DIM   # 2176
MLP_HIDDEN = 4 * N_EMBD      # 8704
VOCAB = 65536
LOGIT_CAP = 15.0
SCALE = 1.0 / math.sqrt(HEAD_DIM)


class Weights:
    """Random-init weights N(0, std) in bf16 on the current device (the architecture of
    src/config.h: 34 layers, d_model 2176, 17 heads x 128, MLP 8704, vocab 65536)."""

    def __init__(self, seed=4, std=0.02, device="cuda"):
        g = torch.Generator(device=device).manual_seed(seed)

        def rnd(*shape):
            return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

        self.embed = rnd(VOCAB, N_EMBD)
        self.layers = []
        for _ in range(N_LAYER):
            self.layers.append(dict(q=rnd(N_EMBD, N_EMBD), k=rnd(N_EMBD, N_EMBD),
                                    v=rnd(N_EMBD, N_EMBD), o=rnd(N_EMBD, N_EMBD),
                                    up=rnd(MLP_HIDDEN, N_EMBD), down=rnd(N_EMBD, MLP_HIDDEN)))
        self.lm_head = rnd(VOCAB, N_EMBD)


class BatchedEngine:
    """`batch` sequences, each with KV caches of `max_len` rows per layer.  temperature 0 is
    greedy decoding; otherwise each step samples with temperature / top_k / top_p as
    Engine::sample does (src/engine.cpp:62-131), from uniform draws made on the device (torch's
    CUDA generator, seeded with `seed`), so sampling stays inside the captured step."""

    def __init__(self, weights, batch, max_len, device="cuda", temperature=0.0, top_k=50,
                 top_p=0.9, seed=None):
        self.w, self.B, self.max_len = weights, batch, max_len
        self.temperature, self.top_k, self.top_p = float(temperature), int(top_k), float(top_p)
        if seed is not None:
            torch.cuda.manual_seed(seed)
        self.uniforms = torch.zeros(batch, dtype=torch.float32, device=device)
        attn.init_rope_tables()
        self._alloc_caches(device)
        self.kv_len = torch.zeros(batch, dtype=torch.int32, device=device)
        self.ws = torch.zeros(attn.decode_workspace_bytes(batch, max_len, N_HEAD),
                              dtype=torch.uint8, device=device)
        self.tok = torch.zeros(batch, dtype=torch.int32, device=device)  # next input token
        # 1 for a slot holding a live sequence: only those lengths advance in a decode step
        self.active = torch.zeros(batch, dtype=torch.int32, device=device)
        # decode-step GEMM operands: fused [q; k; v] weights and the activations
        self.wqkv = [torch.cat([l["q"], l["k"], l["v"]], 0) for l in weights.layers]
        bf = dict(dtype=torch.bfloat16, device=device)
        self.x = torch.zeros((batch, N_EMBD), **bf)           # residual stream
        self.qkv = torch.zeros((3, batch, N_EMBD), **bf)      # q, k, v (pre-RoPE)
        self.a = torch.zeros((batch, N_EMBD), **bf)           # attention output
        self.h = torch.zeros((batch, MLP_HIDDEN), **bf)       # ReLU^2 of the MLP up projection
        self.logits = torch.zeros((batch, VOCAB), **bf)
        self.graph = None

    def _alloc_caches(self, device):
        """One K and one V slab per layer, [batch, max_len, heads, 128], and device arrays of the
        per-sequence bases for the batched decode kernel."""
        shape = (self.B, self.max_len, N_HEAD, HEAD_DIM)
        self.k = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(N_LAYER)]
        self.v = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(N_LAYER)]
        row = self.max_len * N_HEAD * HEAD_DIM * 2

        def table(t):
            return torch.tensor([t.data_ptr() + b * row for b in range(self.B)],
                                dtype=torch.int64, device=device)

        self.k_tab = [table(t) for t in self.k]
        self.v_tab = [table(t) for t in self.v]

    # ------------------------------------------------------------------ cache access
    def _prompt_attention(self, i, b, q, k, v, P, a):
        """Layer i, one sequence in slot b: RoPE + QK-norm + append of its P rows, attention."""
        attn.rope_qknorm_append(q, k, v, self.k[i][b], self.v[i][b], P, N_HEAD, 0)
        attn.flash_attention(a, q, self.k[i][b], self.v[i][b], P, P, N_HEAD, SCALE, 0)

    def _prompt_attention_all(self, i, q, k, v, P, a):
        """Layer i, every slot's prompt of P rows (rows b*P.. of q, k, v)."""
        stride = self.max_len * N_HEAD * HEAD_DIM
        attn.rope_qknorm_append_batched(q, k, v, self.k[i], self.v[i], stride, self.B, P, N_HEAD, 0)
        offs = torch.zeros(self.B, dtype=torch.int32, device=q.device)
        attn.prefill_attention_batched(a, q, self.k[i], self.v[i], stride, self.max_len, offs, P,
                                       N_HEAD, SCALE)

    def _decode_attention(self, i, a, qkv):
        # right after the Q/K/V GEMM, which writes no cache: the attention CTAs may start
        # loading cache rows while it finishes
        attn.decode_attention(a, qkv[0], qkv[1], qkv[2], self.k_tab[i], self.v_tab[i],
                              self.kv_len, N_HEAD, SCALE, self.max_len, self.ws, overlap=True)

    # ------------------------------------------------------------------ prompt
    def _prompt_layers(self, tokens, attention):
        """The prompt pass's layers over rows = tokens (int64 [R]); attention(i, q, k, v, a)
        runs layer i's attention.  Returns the residual stream [R, N_EMBD] after the last
        layer.  Per layer (src/model.cpp:101-154): Q/K/V from RMSNorm(x) in one GEMM pass,
        attention, output projection + residual in place, MLP up from RMSNorm(x) with ReLU^2,
        MLP down + residual in place."""
        w = self.w
        R = int(tokens.numel())
        bf = dict(dtype=torch.bfloat16, device=tokens.device)
        x = torch.empty((R, N_EMBD), **bf)
        G.embed_rmsnorm(x, w.embed, tokens.to(torch.int32))  # embedding + RMSNorm (:158-162)
        qkv = torch.empty((3, R, N_EMBD), **bf)
        a = torch.empty((R, N_EMBD), **bf)
        h = torch.empty((R, MLP_HIDDEN), **bf)
        for i, l in enumerate(w.layers):
            G.gemm(qkv, x, self.wqkv[i], flags=G.NORM_INPUT, seg_cols=N_EMBD)
            attention(i, qkv[0], qkv[1], qkv[2], a)
            G.gemm(x, a, l["o"], residual=x)
            G.gemm(h, x, l["up"], flags=G.NORM_INPUT | G.RELU2)
            G.gemm(x, h, l["down"], residual=x)
        return x

    def _first_tokens(self, last):
        """Greedy first token of each row of `last` [B, N_EMBD]: final RMSNorm, LM head and
        tanh cap (src/model.cpp:170-177) on the skinny GEMM, then the device argmax."""
        logits = torch.empty((last.shape[0], VOCAB), dtype=torch.bfloat16, device=last.device)
        G.gemm_skinny(logits, last.contiguous(), self.w.lm_head, flags=G.NORM_INPUT | G.TANH_CAP,
                      cap=LOGIT_CAP)
        first = torch.empty(last.shape[0], dtype=torch.int32, device=last.device)
        G.argmax_rows(first, logits)
        return first

    def _prompt_pass(self, b, prompt):
        """Prompt pass of one sequence into slot b's caches (rows [0, P)); returns its first
        generated token (greedy, as the reference's first step, src/engine.cpp:37-62)."""
        P = int(prompt.numel())
        assert 0 < P < self.max_len
        x = self._prompt_layers(prompt.reshape(-1),
                                lambda i, q, k, v, a: self._prompt_attention(i, b, q, k, v, P, a))
        return self._first_tokens(x[-1:])[0]

    def prefill(self, prompts):
        """prompts: int64 [B, P] token ids; fills the caches of every slot and sets the first
        generated token of every sequence (returned, and kept as the next decode input).
        All B sequences go through each layer together: the GEMMs run on B*P rows, the RoPE +
        QK-norm + append pass writes each slot's cache rows [0, P), and one batched prefill
        attention launch covers every sequence."""
        B, P = prompts.shape
        assert B == self.B and P < self.max_len
        x = self._prompt_layers(prompts.reshape(-1),
                                lambda i, q, k, v, a: self._prompt_attention_all(i, q, k, v, P, a))
        first = self._first_tokens(x.view(B, P, N_EMBD)[:, -1])
        self.kv_len.fill_(P)
        self.tok.copy_(first)
        self.active.fill_(1)
        return first

    # ------------------------------------------------------------------ continuous batching
    def admit(self, slot, prompt):
        """Starts a new sequence in `slot` between decode steps (continuous batching): its
        prompt pass runs now, its length and next token are set on the device, and the next
        step (graph replay included) advances it with the others.  Returns its first token."""
        first = self._prompt_pass(slot, prompt)
        self.kv_len[slot] = int(prompt.numel())
        self.tok[slot] = first
        self.active[slot] = 1
        return first

    def retire(self, slot):
        """Frees `slot`: its length stops advancing (its rows are recomputed and ignored until a
        new sequence is admitted there)."""
        self.active[slot] = 0

    # ------------------------------------------------------------------ decode
    def _decode_body(self):
        """One greedy step for the whole batch: consumes self.tok, writes the next tokens back
        into self.tok.  Static shapes, device-side lengths: safe to capture."""
        w, x, qkv, a, h = self.w, self.x, self.qkv, self.a, self.h
        self.kv_len.add_(self.active)  # a live slot's new token sits at row kv_len - 1
        G.embed_rmsnorm(x, w.embed, self.tok)  # embedding + RMSNorm (:158-162)
        for i, l in enumerate(w.layers):
            # RMSNorm -> Q/K/V (src/model.cpp:110-116)
            G.gemm_skinny(qkv, x, self.wqkv[i], flags=G.NORM_INPUT, seg_cols=N_EMBD)
            self._decode_attention(i, a, qkv)
            G.gemm_skinny(x, a, l["o"], residual=x)                      # :139
            G.gemm_skinny(h, x, l["up"], flags=G.NORM_INPUT | G.RELU2)  # :146-150
            G.gemm_skinny(x, h, l["down"], residual=x)                   # :153
        # final RMSNorm, LM head, soft cap (:170-177); logits [B, VOCAB] kept for inspection
        G.gemm_skinny(self.logits, x, w.lm_head, flags=G.NORM_INPUT | G.TANH_CAP, cap=LOGIT_CAP)
        if self.temperature == 0.0:
            G.argmax_rows(self.tok, self.logits)  # greedy choice (src/engine.cpp:88-95)
        else:
            torch.rand(self.B, out=self.uniforms)
            G.sample_rows(self.tok, self.logits, self.temperature, self.top_k, self.top_p,
                          self.uniforms)

    def capture(self):
        """Capture one decode step in a CUDA graph (after one eager warm-up step, which also
        performs every per-device set-up outside the capture).  The warm-up step advances
        the sequences like any other step."""
        self._decode_body()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._decode_body()
        return self.tok.clone()

    def step(self):
        """One decode step (graph replay if captured); returns the new tokens (device)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._decode_body()
        return self.tok


class PagedEngine(BatchedEngine):
    """BatchedEngine over a paged KV cache: per layer one K and one V pool of `num_pages` pages of
    `page_rows` rows (a multiple of 128), shared by all slots, and one device page table
    [batch, pages_per_seq] used by every layer.  A host-side allocator hands a slot the pages
    its prompt needs when it is admitted, one more page whenever a decode step is about to write
    the first row of a new page, and takes them all back when the slot retires, so the cache
    holds only the live sequences' rows (num_pages may be far below batch * max_len /
    page_rows).  The attention calls are the library's paged forms (nc_rope_qknorm_append_paged and
    its batched form over the device page table, nc_prefill_attention_paged,
    nc_decode_attention_paged); everything else is BatchedEngine's.
    A retired slot's length is set to 0, so a decode step reads and writes none of its old pages.
    """

    def __init__(self, weights, batch, max_len, page_rows=128, num_pages=None, **kw):
        assert page_rows % 128 == 0
        self.page_rows = page_rows
        self.pages_per_seq = -(-max_len // page_rows)
        self.num_pages = num_pages or batch * self.pages_per_seq
        super().__init__(weights, batch, max_len, **kw)

    def _alloc_caches(self, device):
        shape = (self.num_pages, self.page_rows, N_HEAD, HEAD_DIM)
        self.k = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(N_LAYER)]
        self.v = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(N_LAYER)]
        self.page_table = torch.full((self.B, self.pages_per_seq), -1, dtype=torch.int32,
                                     device=device)
        self.free_pages = list(range(self.num_pages - 1, -1, -1))
        self.pages = [[] for _ in range(self.B)]   # page ids of each slot, in position order
        self.host_len = [0] * self.B               # rows written per slot (host mirror)

    # ------------------------------------------------------------------ page allocator
    def _map_rows(self, slot, n_rows):
        """Makes sure slot's pages cover rows [0, n_rows)."""
        while len(self.pages[slot]) * self.page_rows < n_rows:
            if not self.free_pages:
                raise RuntimeError("paged KV cache: out of pages")
            pid = self.free_pages.pop()
            self.page_table[slot, len(self.pages[slot])] = pid
            self.pages[slot].append(pid)

    def _release(self, slot):
        self.free_pages.extend(reversed(self.pages[slot]))
        self.pages[slot] = []
        self.page_table[slot].fill_(-1)

    def pages_in_use(self):
        return self.num_pages - len(self.free_pages)

    # ------------------------------------------------------------------ cache access
    def _prompt_attention(self, i, b, q, k, v, P, a):
        attn.rope_qknorm_append_paged(q, k, v, self.k[i], self.v[i], self.pages[b], P, N_HEAD, 0)
        offs = torch.zeros(1, dtype=torch.int32, device=q.device)
        attn.prefill_attention_paged(a, q, self.k[i], self.v[i], self.page_table[b:b + 1], offs,
                                     P, N_HEAD, SCALE)

    def _prompt_attention_all(self, i, q, k, v, P, a):
        attn.rope_qknorm_append_paged_batched(q, k, v, self.k[i], self.v[i], self.page_table, P,
                                              N_HEAD, 0)
        offs = torch.zeros(self.B, dtype=torch.int32, device=q.device)
        attn.prefill_attention_paged(a, q, self.k[i], self.v[i], self.page_table, offs, P,
                                     N_HEAD, SCALE)

    def _decode_attention(self, i, a, qkv):
        attn.decode_attention_paged(a, qkv[0], qkv[1], qkv[2], self.k[i], self.v[i],
                                    self.page_table, self.kv_len, N_HEAD, SCALE, self.max_len,
                                    self.ws)

    # ------------------------------------------------------------------ slots and steps
    def prefill(self, prompts):
        B, P = prompts.shape
        for b in range(B):
            self._release(b)
            self._map_rows(b, P)
            self.host_len[b] = P
        return super().prefill(prompts)

    def admit(self, slot, prompt):
        P = int(prompt.numel())
        self._release(slot)
        self._map_rows(slot, P)
        self.host_len[slot] = P
        return super().admit(slot, prompt)

    def retire(self, slot):
        super().retire(slot)
        self.kv_len[slot] = 0  # no decode step touches the slot's (released) pages
        self.host_len[slot] = 0
        self._release(slot)

    def _before_step(self):
        """Maps the page each live slot's next row falls in, then advances the host mirror."""
        for b in range(self.B):
            if self.pages[b]:  # live slot
                self._map_rows(b, self.host_len[b] + 1)
                self.host_len[b] += 1

    def capture(self):
        self._before_step()  # capture() runs one eager step first
        return super().capture()

    def step(self):
        self._before_step()
        return super().step()

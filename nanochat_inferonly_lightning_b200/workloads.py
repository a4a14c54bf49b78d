"""Synthetic workloads at the shapes of the reference engine's attention path.

Shapes, seeds and the algorithmic work that throughput figures are computed from:
  cfg1  decode, 1 sequence, query at position 511, 512 cached keys          (HBM bytes)
  cfg2  causal prefill, 1 sequence, 2048 positions                          (FLOPs)
  cfg3  decode, 64 sequences, kv_len ~ U[1, 2048] (torch seed 2)            (HBM bytes)
  cfg4  chunked prefill, 4 sequences, 512 queries at offset 1536            (FLOPs)
Model geometry: 17 heads x 128 (src/config.h:9-12).  Normal draws come from a seeded CPU
torch.Generator, fp32 then cast to bf16, in the order Q, K, V, then cache contents.
"""
import torch

HEADS = 17
HEAD_DIM = 128
ROW = HEADS * HEAD_DIM  # elements per (position) row of Q/K/V/cache/out
SCALE = 1.0 / (128 ** 0.5)  # src/model.cpp:134 uses 1/sqrtf(HEAD_DIM)


def randn_bf16(shape, gen):
    return torch.randn(shape, generator=gen, dtype=torch.float32).to(torch.bfloat16)


def causal_flops(seq_q, kv_offset, heads=HEADS, head_dim=HEAD_DIM):
    """2 (QK^T and PV) x 2 (multiply-add) x heads x head_dim x visible (query, key) pairs, where
    query i (0-based in the chunk) sees kv_offset + i + 1 keys."""
    pairs = seq_q * kv_offset + seq_q * (seq_q + 1) // 2
    return 2 * 2 * heads * head_dim * pairs


def decode_bytes(kv_lens, heads=HEADS, head_dim=HEAD_DIM):
    """K + V rows read for every visible key, plus the bf16 output row of each sequence."""
    row_bytes = heads * head_dim * 2
    return sum(int(l) for l in kv_lens) * row_bytes * 2 + len(kv_lens) * row_bytes


# ---------------------------------------------------------------------------------- cfg1
CFG1_POS = 511
CFG1_LEN = 512


def cfg1_inputs(seed=0):
    """Q [1,17,128] (pre-RoPE), K/V [512,17,128] (K pre-RoPE), seed 0."""
    g = torch.Generator().manual_seed(seed)
    q = randn_bf16((1, HEADS, HEAD_DIM), g)
    k = randn_bf16((CFG1_LEN, HEADS, HEAD_DIM), g)
    v = randn_bf16((CFG1_LEN, HEADS, HEAD_DIM), g)
    return q, k, v


def cfg1_decode_case(seed=0):
    """cfg1 as the decode step the benchmark times, from cfg1_inputs(seed): the new token at
    position 511 (q, k_new, v_new [1,17,128], pre-RoPE) and the caches [512,17,128] holding the
    keys and values of positions 0..510 (row 511 zero: the step appends the new token there).
    The cache keys are pre-RoPE here: callers apply RoPE + QK-norm to rows 0..510 at positions
    0..510 with their own kernel, as a model's earlier steps would have.  CPU tensors."""
    q, k, v = cfg1_inputs(seed)
    n = CFG1_LEN - 1
    kc = torch.zeros((CFG1_LEN, HEADS, HEAD_DIM), dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kc[:n] = k[:n]
    vc[:n] = v[:n]
    return q, k[n:], v[n:], kc, vc


CFG1_BYTES = decode_bytes([CFG1_LEN])  # 4,460,800


# ---------------------------------------------------------------------------------- cfg2
CFG2_SEQ = 2048


def cfg2_inputs(seq=CFG2_SEQ, seed=1):
    g = torch.Generator().manual_seed(seed)
    q = randn_bf16((seq, HEADS, HEAD_DIM), g)
    k = randn_bf16((seq, HEADS, HEAD_DIM), g)
    v = randn_bf16((seq, HEADS, HEAD_DIM), g)
    return q, k, v


CFG2_FLOPS = causal_flops(CFG2_SEQ, 0)  # 18,262,523,904


# ---------------------------------------------------------------------------------- cfg3
CFG3_BATCH = 64
CFG3_MAX = 2048


def cfg3_kv_lens():
    """kv_len per sequence: torch.randint(1, 2049, (64,)) with seed 2 (sum 63,344)."""
    g = torch.Generator().manual_seed(2)
    return [int(x) for x in torch.randint(1, CFG3_MAX + 1, (CFG3_BATCH,), generator=g)]


def cfg3_bytes(kv_lens=None):
    return decode_bytes(kv_lens if kv_lens is not None else cfg3_kv_lens())


def decode_batch_raw(lens, seed, device="cuda"):
    """A decode step over independent sequences (cfg3 and the like), drawn N(0,1) from a torch
    generator on `device` seeded with `seed`, in this order: per sequence its K cache then its
    V cache ([L_i,17,128]), then the new tokens' q, k_new, v_new ([B,17,128], pre-RoPE).  The
    cache keys are pre-RoPE: callers apply RoPE + QK-norm at positions 0.. with their own kernel
    (rows up to L_i - 2 are read; row L_i - 1 receives the appended new key)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def rnd(shape):
        return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)

    kcs, vcs = [], []
    for L in lens:
        kcs.append(rnd((L, HEADS, HEAD_DIM)))
        vcs.append(rnd((L, HEADS, HEAD_DIM)))
    B = len(lens)
    q = rnd((B, HEADS, HEAD_DIM))
    kn = rnd((B, HEADS, HEAD_DIM))
    vn = rnd((B, HEADS, HEAD_DIM))
    return q, kn, vn, kcs, vcs


# ---------------------------------------------------------------------------------- cfg4
CFG4_BATCH = 4
CFG4_OFFSET = 1536
CFG4_CHUNK = 512
CFG4_FLOPS = CFG4_BATCH * causal_flops(CFG4_CHUNK, CFG4_OFFSET)  # 31,952,732,160


def cfg4_chunk_inputs(batch=CFG4_BATCH, chunk=CFG4_CHUNK, seed=3):
    """Chunk Q/K/V [batch, chunk, 17, 128] (pre-RoPE), seed 3."""
    g = torch.Generator().manual_seed(seed)
    q = randn_bf16((batch, chunk, HEADS, HEAD_DIM), g)
    k = randn_bf16((batch, chunk, HEADS, HEAD_DIM), g)
    v = randn_bf16((batch, chunk, HEADS, HEAD_DIM), g)
    return q, k, v


def cfg4_cache_raw(n, rows=CFG4_OFFSET + CFG4_CHUNK, seed=30, device="cuda"):
    """K and V cache slabs [n, rows, 17, 128] for the chunked prefill, N(0,1) from a torch
    generator on `device` (K slab drawn first).  Rows [0, 1536) stand for the cached prefix:
    callers apply RoPE + QK-norm to their keys at positions 0..1535 with their own kernel; the
    chunk's append writes rows [1536, 2048)."""
    g = torch.Generator(device=device).manual_seed(seed)
    kslab = torch.randn((n, rows, HEADS, HEAD_DIM), generator=g, device=device).to(torch.bfloat16)
    vslab = torch.randn((n, rows, HEADS, HEAD_DIM), generator=g, device=device).to(torch.bfloat16)
    return kslab, vslab


def shard(n_items, rank, world):
    """Contiguous, as-even-as-possible share of n_items for `rank` of `world`: [start, stop)."""
    base, rem = divmod(n_items, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_weighted(weights, rank, world):
    """Contiguous share [start, stop) of the items for `rank` of `world`, with the cut points
    placed so that each rank's sum of weights (a sequence's KV length: the bytes its decode
    streams) is as close as possible to an equal share: cut r goes at the first prefix whose
    sum reaches r/world of the total, or just before it when that is strictly closer.  Every rank gets at
    least one item when there are at least `world` items."""
    n = len(weights)
    if world <= 1 or n == 0:
        return (0, n) if rank == 0 or world <= 1 else (n, n)
    total = float(sum(weights))
    prefix = [0.0]
    for w in weights:
        prefix.append(prefix[-1] + float(w))
    cuts = [0]
    for r in range(1, world):
        target = total * r / world
        i = next((k for k in range(1, n + 1) if prefix[k] >= target), n)
        if i > 0 and abs(prefix[i - 1] - target) < abs(prefix[i] - target):
            i -= 1
        lo = cuts[-1] + (1 if n >= world else 0)   # at least one item per earlier rank
        hi = n - (world - r if n >= world else 0)  # and one left for every later rank
        cuts.append(min(max(i, lo), hi))
    cuts.append(n)
    return cuts[rank], cuts[rank + 1]


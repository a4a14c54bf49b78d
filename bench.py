"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

Headline (BASELINE.json metric, configs[1]): causal prefill attention TFLOP/s at 2048
positions, 17 heads x 128, bf16.  One step = the fused RoPE + QK-norm + KV-append pass over
Q/K/V followed by the tcgen05 prefill attention kernel, i.e. the whole per-layer attention
path of src/model.cpp:119-136 for a 2048-token prompt.  With N GPUs every rank prefills its
own independent sequence (weak scaling, no collective on the data path).

Also reported on the same line ("extra"): decode HBM GB/s for cfg1 (1 sequence, 512 keys) and
cfg3 (64 sequences, kv_len ~ U[1,2048], sharded over ranks), and chunked-prefill TFLOP/s for
cfg4 (4 sequences x 512 queries at offset 1536, sharded over ranks).

Timing: W untimed warm-up steps, then K steps back to back between two CUDA events on the
launching stream (barrier + synchronize on both sides; the max over ranks is reported).  Every
workload rotates through enough independent input sets that the sets together exceed twice
the L2 (126 MB), so each step starts with its inputs out of L2 without a flush inside the
timed region.  A GPU-side hold spin queued before the start event, long enough to cover the
host's launches of all K steps, keeps host launch latency out of the device timing.  The
attention kernel and the RoPE/append pass are also timed on their own, the same way, for the
roofline.  `e2e` repeats the headline through the public API from pinned host
buffers with the host->device copies of Q/K/V and the device->host copy of the output inside
the timed region, successive steps alternating between two streams so that copies overlap
kernels.

--impl reference runs the same workloads through the reference's own CUDA kernels
(kernels/rope.cu + kernels/flash_attention.cu rebuilt for sm_100a, oracle/_ref) and the
reference's call sequence (two apply_rope_rmsnorm launches, two append copies,
flash_attention per sequence).
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from nanochat_inferonly_lightning_b200 import workloads as W  # noqa: E402

H, D, ROW = W.HEADS, W.HEAD_DIM, W.ROW


# ------------------------------------------------------------------------------ plumbing
class Dist:
    """One process per GPU (RANK / LOCAL_RANK / WORLD_SIZE from the launcher).  Collectives
    are used only outside the timed regions: barriers around them and the max / sum of the
    per-rank results.  backend="gloo" runs the same logic on CPU (tests)."""

    def __init__(self, n_gpus, backend="nccl", timeout_s=120):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}")
        self.device = "cuda" if backend == "nccl" else "cpu"
        if backend == "nccl":
            torch.cuda.set_device(self.local)
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            kw = {"device_id": torch.device("cuda", self.local)} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def _reduce(self, x, op):
        if not self.pg:
            return x
        t = torch.tensor([float(x)], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x):
        return self._reduce(x, self.pg.ReduceOp.MAX if self.pg else None)

    def sum(self, x):
        return self._reduce(x, self.pg.ReduceOp.SUM if self.pg else None)

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Single:
    """A one-rank stand-in for Dist (reference arm)."""

    def __init__(self, local):
        self.rank, self.world, self.local = 0, 1, local

    def barrier(self):
        pass

    def max(self, x):
        return x

    def sum(self, x):
        return x

    def close(self):
        pass


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return {"hbm": j["hbm_gbs"], "tflops": j["bf16_tflops"], "src": "measured"}
    return {"hbm": 6650.0, "tflops": 1590.0, "src": "fallback"}


def load_traffic():
    """Per-launch DRAM bytes of the dominant kernels from a committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except ValueError:
            return {}
    return {}


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms while a region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index, log_dir=None):
        self.idx = device_index
        self.proc = None
        if log_dir is None:
            import tempfile

            log_dir = tempfile.gettempdir()
        self.path = os.path.join(log_dir, f"nc_bench_clocks_rank{device_index}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


L2_BYTES = 126 << 20
# A GPU-side spin (torch's _sleep kernel) queued just before the start event holds the stream
# while the host enqueues the K timed steps, so the events bracket device execution and not
# the host's launch latency (the blocking-kernel method of nvbench): at least ~0.5 ms, plus
# ~50 us of spin per step, well above the host's cost of enqueueing a step.  The e2e figure,
# which goes through the host API with host buffers, includes the host cost.
HOLD_CYCLES = 1_000_000
HOLD_CYCLES_PER_STEP = 100_000


def input_sets(set_bytes):
    """How many independent copies of a workload's inputs to rotate through so that all of them
    together exceed twice the L2: a step's inputs were last touched at least 2x L2 of other
    traffic earlier, so they start out of L2.  A set of 2x L2 or more is its own rotation."""
    set_bytes = max(int(set_bytes), 1)
    if set_bytes >= 2 * L2_BYTES:
        return 1
    return -(-2 * L2_BYTES // set_bytes) + 1


class Stepper:
    """Runs W warm-up steps, then K steps back to back between two events, and returns the mean
    per-step device time in ms.  The step callable rotates through its own input sets."""

    def __init__(self, dist):
        self.dist = dist

    def run(self, step, K, Wm):
        for _ in range(Wm):
            step()
        torch.cuda.synchronize()
        self.dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(max(HOLD_CYCLES, K * HOLD_CYCLES_PER_STEP))
        e0.record()
        for _ in range(K):
            step()
        e1.record()
        torch.cuda.synchronize()
        self.dist.barrier()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / K


# ------------------------------------------------------------------------------ workloads
def prep_normed(impl, x, start_pos):
    """RoPE + QK-norm in place (input setup, untimed) with the arm's own kernel, so the
    reference arm never loads the product library."""
    if impl.kind == "nc":
        impl.nc.apply_rope_rmsnorm(x, x.shape[0], H, start_pos)
    else:
        assert impl.ref.ref_apply_rope_rmsnorm(ptr(x), x.shape[0], H, start_pos, stream()) == 0


class Impl:
    """The product path (nc_*) or the reference kernels (ref_*), same call shapes."""

    def __init__(self, kind):
        self.kind = kind
        if kind == "nc":
            import nanochat_inferonly_lightning_b200 as nc

            self.nc = nc
            self.lib = nc.load()
            nc.init_rope_tables()
        else:
            import oracle

            self.ref = oracle.reference_kernels()
            if self.ref is None:
                raise RuntimeError("reference kernels not built (oracle/_ref)")
            assert self.ref.ref_init_rope_tables() == 0

    # one layer's attention for one sequence chunk: RoPE+QK-norm(q,k), append, attention.
    # Returns the number of this library's kernels launched (0 for the reference arm).
    def prologue(self, q, k, v, kc, vc, seq, start):
        if self.kind == "nc":
            st = self.lib.nc_rope_qknorm_append(ptr(q), ptr(k), ptr(v), ptr(kc), ptr(vc), seq, H,
                                                start, stream())
            assert st == 0, st
            return 1
        r = self.ref
        assert r.ref_apply_rope_rmsnorm(ptr(q), seq, H, start, stream()) == 0
        assert r.ref_apply_rope_rmsnorm(ptr(k), seq, H, start, stream()) == 0
        kc[start:start + seq].copy_(k[:seq])
        vc[start:start + seq].copy_(v[:seq])
        return 0

    def attention(self, out, q, kc, vc, seq, start):
        if self.kind == "nc":
            st = self.lib.nc_flash_attention(ptr(out), ptr(q), ptr(kc), ptr(vc), seq, start + seq,
                                             H, W.SCALE, start, stream())
            assert st == 0, st
            return 1
        assert self.ref.ref_flash_attention(ptr(out), ptr(q), ptr(kc), ptr(vc), seq, start + seq,
                                            H, float(W.SCALE), start, stream()) == 0
        return 0

    def prefill_step(self, out, q, k, v, kc, vc, seq, start):
        return self.prologue(q, k, v, kc, vc, seq, start) + self.attention(out, q, kc, vc, seq, start)


def bench_prefill(impl, dist, stepper, K, Wm, peaks, traffic, e2e=True):
    q0, k0, v0 = (t.cuda() for t in W.cfg2_inputs(seed=1 + dist.rank))
    S = W.CFG2_SEQ
    # Per set: q, k, v, the K/V cache and the output, 8.9 MB each.  The RoPE pass normalises q
    # in place, so a set's q is re-normalised on each reuse: unit RMS and rotated, the same
    # statistics and the same work every time.
    R = input_sets(6 * q0.numel() * 2)
    sets = []
    for _ in range(R):
        kc = torch.zeros((S, H, D), dtype=torch.bfloat16, device="cuda")
        sets.append((q0.clone(), k0.clone(), v0.clone(), kc, torch.zeros_like(kc),
                     torch.empty((S, ROW), dtype=torch.bfloat16, device="cuda")))
    it = [0]
    launches = [0]

    def nxt():
        s_ = sets[it[0] % R]
        it[0] += 1
        return s_

    def step():
        q, k, v, kc, vc, out = nxt()
        launches[0] += impl.prefill_step(out, q, k, v, kc, vc, S, 0)

    def attn():
        q, k, v, kc, vc, out = nxt()
        impl.attention(out, q, kc, vc, S, 0)

    def pro():
        q, k, v, kc, vc, out = nxt()
        impl.prologue(q, k, v, kc, vc, S, 0)

    # The whole step (the attention kernel's setup may overlap the RoPE pass: programmatic
    # dependent launch), then each kernel on its own for the roofline.
    t_step = dist.max(stepper.run(step, K, Wm))
    launches_timed = (launches[0] // (K + Wm)) * K
    t_attn = dist.max(stepper.run(attn, K, Wm))
    t_pro = dist.max(stepper.run(pro, K, Wm))
    flops_rank = W.CFG2_FLOPS
    total = dist.sum(flops_rank)
    res = {
        "value": total / (t_step * 1e-3) / 1e12,
        "ms_per_step": t_step,
        "attn_kernel_ms": t_attn,
        "prologue_ms": t_pro,
        "input_sets": R,
        "gpu_launches": launches_timed,
        "roofline": {
            "bound": "tensor", "achieved": flops_rank / (t_attn * 1e-3) / 1e12,
            "peak": peaks["tflops"], "unit": "TFLOP/s",
            "frac": flops_rank / (t_attn * 1e-3) / 1e12 / peaks["tflops"],
            "traffic": traffic.get("prefill_kernel_cfg2") if impl.kind == "nc" else None,
            "kernel": "prefill_kernel (tcgen05)" if impl.kind == "nc" else "flash_attention_kernel",
            "peak_src": peaks["src"] + " bf16 burst",
        },
    }
    if e2e:
        res["e2e"] = bench_prefill_e2e(impl, dist, K, Wm, q0, k0, v0)
    return res


def bench_prefill_e2e(impl, dist, K, Wm, q0, k0, v0):
    """Same step through the public API from pinned host buffers: every step copies its Q/K/V
    host->device, runs the attention path and copies its output device->host, all inside the
    timed region.  Successive steps alternate between two CUDA streams, each with its own
    device buffers, so one step's host->device copy overlaps the previous step's kernels and
    its device->host copy (the copy engines and the SMs work at the same time; the host link
    is the bound)."""
    S = W.CFG2_SEQ
    hq, hk, hv = (t.cpu().pin_memory() for t in (q0, k0, v0))
    lanes = []
    for _ in range(2):
        kc = torch.zeros((S, H, D), dtype=torch.bfloat16, device="cuda")
        lanes.append((torch.cuda.Stream(), torch.empty_like(q0), torch.empty_like(k0),
                      torch.empty_like(v0), kc, torch.zeros_like(kc),
                      torch.empty((S, ROW), dtype=torch.bfloat16, device="cuda"),
                      torch.empty((S, ROW), dtype=torch.bfloat16).pin_memory()))
    it = [0]

    def step():
        st, q, k, v, kc, vc, out, hout = lanes[it[0] % 2]
        it[0] += 1
        with torch.cuda.stream(st):
            q.copy_(hq, non_blocking=True)
            k.copy_(hk, non_blocking=True)
            v.copy_(hv, non_blocking=True)
            impl.prefill_step(out, q, k, v, kc, vc, S, 0)
            hout.copy_(out, non_blocking=True)

    for _ in range(Wm):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    main = torch.cuda.current_stream()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record(main)
    for ln in lanes:
        ln[0].wait_stream(main)
    for _ in range(K):
        step()
    for ln in lanes:
        main.wait_stream(ln[0])
    e.record(main)
    torch.cuda.synchronize()
    dist.barrier()
    t = dist.max(s.elapsed_time(e) / K)
    bi = 3 * S * ROW * 2
    bo = S * ROW * 2
    return {"value": dist.sum(W.CFG2_FLOPS) / (t * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": t, "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
            "pipelining": "steps alternate between two CUDA streams (copies overlap kernels)"}


def build_decode_batch(impl, lens, seed):
    """workloads.decode_batch_raw's step (caches drawn N(0,1) on the device), with each cache's
    keys RoPE + QK-normalised at positions 0.. by the arm's own kernel."""
    q, kn, vn, kcs, vcs = W.decode_batch_raw(lens, seed)
    for kc in kcs:
        prep_normed(impl, kc, 0)
    return q, kn, vn, kcs, vcs


def build_cfg1(impl, seed):
    """workloads.cfg1_decode_case(seed) on the device: the new token at position 511 and the
    caches' 511 earlier keys RoPE + QK-normalised by the arm's own kernel."""
    q, kn, vn, kc, vc = (t.cuda() for t in W.cfg1_decode_case(seed))
    prep_normed(impl, kc[:W.CFG1_LEN - 1], 0)
    return q, kn, vn, [kc], [vc]


def bench_decode(impl, dist, stepper, K, Wm, peaks, traffic, lens_all, name):
    # Independent sequences, cut into contiguous shares of about equal KV bytes (each rank's
    # decode time follows the bytes it streams, not its sequence count).
    a, b = W.shard_weighted(lens_all, dist.rank, dist.world)
    lens = lens_all[a:b]
    bytes_rank = W.decode_bytes(lens) if lens else 0
    t_ms = 0.0
    launches = 0
    if lens:
        # Independent input sets (caches + new tokens), rotated so that each step's caches start
        # out of L2; cfg3 on one GPU already exceeds 2x L2 and needs one set.
        R = input_sets(bytes_rank)
        B = len(lens)
        mx = max(lens)
        ws = (torch.zeros(impl.nc.decode_workspace_bytes(B, mx, H), dtype=torch.uint8,
                          device="cuda") if impl.kind == "nc" else None)
        set_steps = []
        for rs in range(R):
            # cfg1: set 0 is BASELINE's seed-0 draw; cfg3: the device draw seeded 2 (rank 0)
            if name == "cfg1":
                q, kn, vn, kcs, vcs = build_cfg1(impl, seed=1000 * rs)
            else:
                q, kn, vn, kcs, vcs = build_decode_batch(impl, lens, seed=2 + dist.rank + 1000 * rs)
            out = torch.empty((B, ROW), dtype=torch.bfloat16, device="cuda")
            if impl.kind == "nc":
                kp = torch.tensor([t.data_ptr() for t in kcs], dtype=torch.int64, device="cuda")
                vp = torch.tensor([t.data_ptr() for t in vcs], dtype=torch.int64, device="cuda")
                lt = torch.tensor(lens, dtype=torch.int32, device="cuda")
                lib = impl.lib

                def step_set(out=out, q=q, kn=kn, vn=vn, kp=kp, vp=vp, lt=lt, keep=(kcs, vcs)):
                    st = lib.nc_decode_attention(ptr(out), ptr(q), ptr(kn), ptr(vn), ptr(kp),
                                                 ptr(vp), ptr(lt), B, H, W.SCALE, mx, 0, ptr(ws),
                                                 ws.numel(), stream())
                    assert st == 0, st
            else:
                r = impl.ref
                qs = q.clone()
                ks = kn.clone()

                def step_set(out=out, q=q, kn=kn, vn=vn, kcs=kcs, vcs=vcs, qs=qs, ks=ks):
                    qs.copy_(q)
                    ks.copy_(kn)
                    for i, L in enumerate(lens):
                        qi = qs[i:i + 1]
                        ki = ks[i:i + 1]
                        assert r.ref_apply_rope_rmsnorm(ptr(qi), 1, H, L - 1, stream()) == 0
                        assert r.ref_apply_rope_rmsnorm(ptr(ki), 1, H, L - 1, stream()) == 0
                        kcs[i][L - 1:L].copy_(ki)
                        vcs[i][L - 1:L].copy_(vn[i:i + 1])
                        assert r.ref_flash_attention(ptr(out[i:i + 1]), ptr(qi), ptr(kcs[i]),
                                                     ptr(vcs[i]), 1, L, H, float(W.SCALE), L - 1,
                                                     stream()) == 0
            set_steps.append(step_set)
        launches = 1 if impl.kind == "nc" else 0
        it = [0]

        def step():
            set_steps[it[0] % R]()
            it[0] += 1

        t_ms = stepper.run(step, K, Wm)
    else:
        R = 0
        stepper.run(lambda: None, K, Wm)
    t = dist.max(t_ms)
    total = dist.sum(bytes_rank)
    gbs = total / (t * 1e-3) / 1e9 if t > 0 else 0.0
    rank_gbs = bytes_rank / (t_ms * 1e-3) / 1e9 if t_ms > 0 else 0.0
    return {
        "value": gbs, "unit": "GB/s", "ms_per_step": t, "sequences": len(lens_all),
        "bytes": W.decode_bytes(lens_all), "gpu_launches_per_step": launches,
        "timing": f"back-to-back steps over {R} rotating input set(s) (> 2x L2 in total)",
        "roofline": {"bound": "hbm", "achieved": rank_gbs, "peak": peaks["hbm"], "unit": "GB/s",
                     "frac": rank_gbs / peaks["hbm"],
                     "traffic": traffic.get(f"decode_kernel_{name}") if impl.kind == "nc" else None,
                     "peak_src": peaks["src"]},
    }


def bench_cfg5(dist):
    """cfg5: end-to-end greedy generation on the full 2.2B architecture with random N(0, 0.02)
    weights (seed 4), 8 sequences per GPU, 256-token prompts (uniform ids), 256 decode steps.
    Each decode step replays one CUDA graph for the whole batch, all on this library
    (nanochat_inferonly_lightning_b200/engine.py): per layer the fused Q/K/V GEMM (RMSNorm
    fused), the decode attention (RoPE, QK-norm, append, split-KV), the output projection +
    residual, the MLP up projection (RMSNorm, ReLU^2 fused) and down projection + residual on
    the skinny tcgen05 GEMM, then the LM head (RMSNorm, tanh cap fused), with the embedding
    gather + RMSNorm and the argmax as library kernels too.  The prompt pass runs eagerly for
    all 8 sequences together, also all on this library (the prompt-pass tcgen05 GEMM nc_gemm,
    the batched RoPE/append pass and the batched prefill attention).  Reported: decode tokens
    per second (whole job), timed with CUDA events over the 256 steps, and the prompt pass time
    (after one untimed warm-up pass)."""
    from nanochat_inferonly_lightning_b200 import engine as E

    batch, prompt_len, steps = 8, 256, 256
    w = E.Weights(seed=4)
    g = torch.Generator().manual_seed(4 + dist.rank)
    prompts = torch.randint(0, E.VOCAB, (batch, prompt_len), generator=g).cuda()
    eng = E.BatchedEngine(w, batch, prompt_len + steps + 8)
    eng.prefill(prompts)  # warm-up: library, cuBLAS and kernel-module set-up (not timed)
    dist.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    eng.prefill(prompts)
    s1.record()
    eng.capture()  # one eager warm-up step, then the capture (not timed)
    toks = torch.empty(steps, batch, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        toks[i].copy_(eng.step())
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    t_dec = dist.max(e0.elapsed_time(e1))
    t_pre = dist.max(s0.elapsed_time(s1))
    n_tok = dist.sum(batch * steps)
    del eng, w
    torch.cuda.empty_cache()
    return {"value": n_tok / (t_dec * 1e-3), "unit": "tok/s (decode)",
            "ms_per_decode_step": t_dec / steps, "prompt_pass_ms": t_pre,
            "sequences_per_gpu": batch, "prompt_len": prompt_len, "decode_steps": steps,
            "timing": "CUDA events around 256 graph replays (whole batch per step); the "
                      "prompt pass (8 sequences together, eager, after one untimed warm-up "
                      "pass) is reported separately",
            "note": "decode step: skinny tcgen05 GEMMs with fused RMSNorm/residual/ReLU^2/"
                    "tanh cap and this library's decode attention; bound by streaming the "
                    "4.15 GB of weights read per step"}


def write_reference_weights(path, seed=4):
    """Seed-4 random weights (engine.Weights, N(0, 0.02) bf16) written in the reference's
    weights.bin layout (src/model.cpp:17-35): embedding, per layer q, k, v, o, MLP up, MLP
    down, then the LM head, raw bf16."""
    from nanochat_inferonly_lightning_b200 import engine as E

    w = E.Weights(seed=seed)
    with open(path, "wb") as f:
        def put(t):
            t.contiguous().view(torch.int16).cpu().numpy().tofile(f)

        put(w.embed)
        for l in w.layers:
            for key in ("q", "k", "v", "o", "up", "down"):
                put(l[key])
        put(w.lm_head)
    del w
    torch.cuda.empty_cache()


def bench_cfg5_reference(dist):
    """cfg5 on the reference's own engine (src/model.cpp + src/engine.cpp with its CUTLASS GEMM
    and its attention kernels, rebuilt for sm_100a into oracle/_ref/libref_model_ref.so): the
    same seed-4 weights, loaded from a weights.bin file by the reference's loader, and the same
    8 prompts, decoded one sequence after another with Engine::generate at temperature 0
    (batch 1, as the reference serves).  Engine::generate synchronises with the host after
    every token, so the figure is wall-clock time around each call: decode tok/s = generated
    tokens after the first / (time of a 256-token generation - time of its prompt pass alone)."""
    import tempfile

    so = os.path.join(ROOT, "oracle", "_ref", "libref_model_ref.so")
    if not os.path.exists(so):
        return {"unavailable": "oracle/_ref/libref_model_ref.so not built"}
    lib = ctypes.CDLL(so)
    vp, ip = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)
    lib.refe_create.restype = vp
    lib.refe_load.argtypes = [vp, ctypes.c_char_p]
    lib.refe_generate_greedy.argtypes = [vp, ip, ctypes.c_int, ctypes.c_int, ip]
    lib.refe_destroy.argtypes = [vp]
    batch, prompt_len, steps = 8, 256, 256
    tmpdir = tempfile.mkdtemp(prefix="nc_ref_weights_")
    path = os.path.join(tmpdir, "weights.bin")
    try:
        write_reference_weights(path)
        e = lib.refe_create()
        if not e or lib.refe_load(e, path.encode()) != 0:
            return {"unavailable": "reference engine failed to load the weights file"}
    finally:
        if os.path.exists(path):
            os.remove(path)
        os.rmdir(tmpdir)
    g = torch.Generator().manual_seed(4 + dist.rank)
    prompts = torch.randint(0, 65536, (batch, prompt_len), generator=g).tolist()
    out = (ctypes.c_int * steps)()
    arr0 = (ctypes.c_int * prompt_len)(*prompts[0])
    lib.refe_generate_greedy(e, arr0, prompt_len, 4, out)  # warm-up (module and cache set-up)
    t_full, t_prompt, n_gen = 0.0, 0.0, 0
    for pr in prompts:
        arr = (ctypes.c_int * prompt_len)(*pr)
        t0 = time.perf_counter()
        lib.refe_generate_greedy(e, arr, prompt_len, 1, out)  # prompt pass + first token
        t1 = time.perf_counter()
        n = lib.refe_generate_greedy(e, arr, prompt_len, steps, out)
        t2 = time.perf_counter()
        t_prompt += t1 - t0
        t_full += t2 - t1
        n_gen += max(n - 1, 0)
    lib.refe_destroy(e)
    torch.cuda.synchronize()
    dec = max(t_full - t_prompt, 1e-9)
    return {"value": n_gen / dec, "unit": "tok/s (decode)",
            "ms_per_decode_step": dec / max(n_gen, 1) * 1e3,
            "prompt_pass_ms": t_prompt / batch * 1e3, "sequences": batch,
            "prompt_len": prompt_len, "decode_steps": steps,
            "timing": "wall clock around Engine::generate (host-synchronous per token), 8 "
                      "sequences one after another, batch 1; decode time = full generation "
                      "minus its prompt pass",
            "engine": "reference src/model.cpp + src/engine.cpp, CUTLASS GEMM (4.5 headers), "
                      "reference attention kernels, sm_100a"}


GEMM_SHAPES = (  # decode-step GEMMs of the full architecture (src/model.cpp:110-177)
    ("qkv", 3 * 2176, 2176, "NORM_INPUT", 2176),
    ("o", 2176, 2176, "RESIDUAL", 0),
    ("up", 8704, 2176, "NORM_INPUT|RELU2", 0),
    ("down", 2176, 8704, "RESIDUAL", 0),
    ("lm_head", 65536, 2176, "NORM_INPUT|TANH_CAP", 0),
)


def bench_gemm(dist, stepper, K, Wm, peaks, traffic, M=8):
    """The skinny tcgen05 GEMM on each decode-step shape at M = 8 rows (the cfg5 batch), with
    its fused epilogue.  A step calls it once per copy of the weight, over enough copies
    (> 2x L2 together) that every call streams its weight from HBM, as in the engine where each
    layer's weights are read once per step.  Calls run back to back from a CUDA graph
    (programmatic dependent launch lets each start streaming while the previous one finishes).  Algorithmic bytes per
    call: the weight N*K*2 plus x, the output and the residual."""
    import nanochat_inferonly_lightning_b200 as nc

    G = nc.gemm
    out = {}
    for name, N, Kd, flag_names, seg in GEMM_SHAPES:
        flags = 0
        for f in flag_names.split("|"):
            flags |= getattr(G, f)
        copies = max(2, -(-int(2.2 * L2_BYTES) // (N * Kd * 2)))
        g = torch.Generator(device="cuda").manual_seed(40 + dist.rank)
        ws = [(torch.randn((N, Kd), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
              for _ in range(copies)]
        x = torch.randn((M, Kd), generator=g, device="cuda").to(torch.bfloat16)
        res = torch.randn((M, N), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        kw = dict(flags=flags & ~G.RESIDUAL, cap=15.0, seg_cols=seg)
        if flags & G.RESIDUAL:
            kw["residual"] = res

        def calls():
            for wt in ws:
                G.gemm_skinny(y, x, wt, **kw)

        # One step = one replay of a CUDA graph of the calls (as the engine replays its decode
        # step), so the host's per-call cost is not in the timed region.
        calls()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                calls()
        torch.cuda.current_stream().wait_stream(side)
        t_ms = dist.max(stepper.run(graph.replay, K, Wm)) / copies  # slowest rank
        del graph
        nbytes = N * Kd * 2 + M * Kd * 2 + M * N * 2 * (2 if flags & G.RESIDUAL else 1)
        gbs = nbytes / (t_ms * 1e-3) / 1e9
        out[name] = {"N": N, "K": Kd, "M": M, "fused": flag_names, "us": t_ms * 1e3,
                     "GB_per_s": gbs, "frac_hbm": gbs / peaks["hbm"],
                     "traffic": traffic.get(f"gemm_skinny_{name}_m8")}
        del ws
        torch.cuda.empty_cache()
    out["peak_src"] = peaks["src"]
    out["timing"] = ("mean per call: K replays of a CUDA graph of one call per weight copy, back "
                     "to back between two CUDA events; weight copies > 2x L2 together; per-GPU "
                     "figure of the slowest rank")
    return out


def bench_prompt_gemm(dist, stepper, K, Wm, peaks, M=2048, shapes=None):
    """The prompt-pass tcgen05 GEMM (nc_gemm) on the four per-layer shapes of the cfg5 prompt
    pass (8 sequences x 256 tokens = 2048 rows) with their fused steps.  Each step runs one
    call per input set, over enough sets (x, weight, out; > 2x L2 together) that every call
    reads its operands from HBM, from one CUDA graph replay.  FLOPs per call: 2*M*N*K."""
    import nanochat_inferonly_lightning_b200 as nc

    G = nc.gemm
    out = {}
    for name, N, Kd, flag_names, seg in (shapes or GEMM_SHAPES[:4]):
        flags = 0
        for f in flag_names.split("|"):
            flags |= getattr(G, f)
        per_set = (N * Kd + M * Kd + M * N) * 2
        sets = max(2, -(-int(2.2 * L2_BYTES) // per_set))
        g = torch.Generator(device="cuda").manual_seed(60 + dist.rank)
        data = [((torch.randn((M, Kd), generator=g, device="cuda")).to(torch.bfloat16),
                 (torch.randn((N, Kd), generator=g, device="cuda") * 0.02).to(torch.bfloat16),
                 torch.randn((M, N), generator=g, device="cuda").to(torch.bfloat16))
                for _ in range(sets)]

        def calls():
            for x, w, y in data:
                # the residual flag adds y in place (out == residual), as the engine does
                G.gemm(y, x, w, residual=y if flags & G.RESIDUAL else None,
                       flags=flags & ~G.RESIDUAL, cap=15.0, seg_cols=seg)

        calls()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                calls()
        torch.cuda.current_stream().wait_stream(side)
        t_ms = dist.max(stepper.run(graph.replay, K, Wm)) / sets
        del graph
        tf = 2.0 * M * N * Kd / (t_ms * 1e-3) / 1e12
        out[name] = {"M": M, "N": N, "K": Kd, "fused": flag_names, "us": t_ms * 1e3,
                     "TFLOP_per_s": tf, "frac_bf16": tf / peaks["tflops"]}
        del data
        torch.cuda.empty_cache()
    out["peak_src"] = peaks["src"]
    out["timing"] = ("mean per call: K replays of a CUDA graph of one call per input set, back "
                     "to back between two CUDA events; input sets > 2x L2 together")
    return out


def bench_chunked(impl, dist, stepper, K, Wm, peaks, traffic):
    a, b = W.shard(W.CFG4_BATCH, dist.rank, dist.world)
    n = b - a
    off, C = W.CFG4_OFFSET, W.CFG4_CHUNK
    t_ms = 0.0
    if n > 0:
        q0, k0, v0 = (t[a:b].cuda() for t in W.cfg4_chunk_inputs())
        rows = off + C
        # Per set: q, k, v, out (n x C rows) and the two cache slabs (n x rows); q is
        # re-normalised in place on reuse (same statistics, same work).
        R = input_sets(n * (4 * C + 2 * rows) * ROW * 2)
        sets = []
        for rs in range(R):
            kslab, vslab = W.cfg4_cache_raw(n, rows, seed=30 + dist.rank + 1000 * rs)
            for i in range(n):
                prep_normed(impl, kslab[i, :off], 0)
            sets.append((q0.clone(), k0.clone(), v0.clone(), kslab, vslab,
                         torch.empty((n, C, ROW), dtype=torch.bfloat16, device="cuda")))
        it = [0]
        if impl.kind == "nc":
            lib = impl.lib
            offs = torch.full((n,), off, dtype=torch.int32, device="cuda")

            def step():
                # one RoPE/QK-norm/append launch for the whole batch of chunks, then one
                # attention launch over it (the reference arm has no batched entry points)
                q, k, v, kslab, vslab, out = sets[it[0] % R]
                it[0] += 1
                st = lib.nc_rope_qknorm_append_batched(ptr(q), ptr(k), ptr(v), ptr(kslab),
                                                       ptr(vslab), rows * ROW, n, C, H, off,
                                                       stream())
                assert st == 0, st
                st = lib.nc_prefill_attention_batched(ptr(out), ptr(q), ptr(kslab), ptr(vslab),
                                                      rows * ROW, rows, ptr(offs), n, C, H,
                                                      W.SCALE, stream())
                assert st == 0, st
        else:
            def step():
                q, k, v, kslab, vslab, out = sets[it[0] % R]
                it[0] += 1
                for i in range(n):
                    impl.prefill_step(out[i], q[i], k[i], v[i], kslab[i], vslab[i], C, off)

        t_ms = stepper.run(step, K, Wm)
    else:
        stepper.run(lambda: None, K, Wm)
    t = dist.max(t_ms)
    flops_rank = n * W.causal_flops(C, off)
    total = dist.sum(flops_rank)
    return {"value": total / (t * 1e-3) / 1e12 if t > 0 else 0.0, "unit": "TFLOP/s",
            "ms_per_step": t, "sequences": W.CFG4_BATCH}


def cpu_baseline_prefill(seconds_hint=20.0):
    """The C oracle (fp32, OpenMP over rows) on a bounded sample of cfg2: the last `rows`
    query rows of the 2048-position causal prefill (the most expensive rows), all 17 heads."""
    import oracle

    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    q, k, v = W.cfg2_inputs()
    qu = q.view(torch.int16).numpy().view(np.uint16)
    ku = k.view(torch.int16).numpy().view(np.uint16)
    vu = v.view(torch.int16).numpy().view(np.uint16)
    rows = 32
    t0 = time.perf_counter()
    oracle.flash_attention(qu[-rows:], ku, vu, rows, 2048, H, W.SCALE, 2048 - rows)
    dt = time.perf_counter() - t0
    # grow the sample toward ~seconds_hint of CPU work (bounded)
    if dt < seconds_hint / 4:
        rows = int(min(2048, max(rows, rows * (seconds_hint / 2) / max(dt, 1e-3))))
        t0 = time.perf_counter()
        oracle.flash_attention(qu[-rows:], ku, vu, rows, 2048, H, W.SCALE, 2048 - rows)
        dt = time.perf_counter() - t0
    flops = 2 * 2 * H * D * sum(2048 - rows + i + 1 for i in range(rows))
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"oracle/nc_oracle.c attention, last {rows} query rows of cfg2 "
                      f"(17 heads, causal over 2048 keys), {dt:.1f} s"}


# ------------------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["nc", "reference"], default="nc")
    ap.add_argument("--no-extra", action="store_true", help="headline only")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU oracle baseline")
    ap.add_argument("--clock-log-dir", default=None,
                    help="directory for the raw nvidia-smi clock samples (default: the system "
                         "temporary directory)")
    ap.add_argument("--only", choices=["prefill", "cfg1", "cfg3", "cfg4", "gemm", "prompt_gemm",
                                       "cfg5"],
                    default=None,
                    help="run one workload only (profiling); implies --no-cpu, no e2e")
    args = ap.parse_args()
    K, Wm = args.steps, max(args.warmup, 3)

    dist = Dist(args.gpus)
    if args.impl == "reference":
        # Rank 0 alone runs the reference arm; the other ranks leave without work.
        rank = dist.rank
        dist.close()
        if rank != 0:
            return
        dist = Single(dist.local)
    impl = Impl("nc" if args.impl == "nc" else "reference")
    peaks = load_peaks()
    traffic = load_traffic()
    stepper = Stepper(dist)

    if args.only:
        fn = {"prefill": lambda: bench_prefill(impl, dist, stepper, K, Wm, peaks, traffic, False),
              "cfg1": lambda: bench_decode(impl, dist, stepper, K, Wm, peaks, traffic,
                                           [W.CFG1_LEN], "cfg1"),
              "cfg3": lambda: bench_decode(impl, dist, stepper, K, Wm, peaks, traffic,
                                           W.cfg3_kv_lens(), "cfg3"),
              "cfg4": lambda: bench_chunked(impl, dist, stepper, K, Wm, peaks, traffic),
              "gemm": lambda: bench_gemm(dist, stepper, K, Wm, peaks, traffic),
              "prompt_gemm": lambda: bench_prompt_gemm(dist, stepper, K, Wm, peaks),
              "cfg5": (lambda: bench_cfg5(dist)) if impl.kind == "nc"
                      else (lambda: bench_cfg5_reference(dist))}[args.only]
        r = fn()
        if dist.rank == 0:
            print(json.dumps({"only": args.only, "impl": args.impl, **r}), flush=True)
        dist.close()
        return
    clocks = ClockSampler(dist.local, args.clock_log_dir)
    clocks.start()
    head = bench_prefill(impl, dist, stepper, K, Wm, peaks, traffic)
    extra = {}
    if not args.no_extra:
        extra["cfg1_decode"] = bench_decode(impl, dist, stepper, K, Wm, peaks, traffic,
                                            [W.CFG1_LEN] if dist.rank == 0 else [], "cfg1") \
            if dist.world == 1 else None
        extra["cfg3_decode"] = bench_decode(impl, dist, stepper, K, Wm, peaks, traffic,
                                            W.cfg3_kv_lens(), "cfg3")
        extra["cfg4_chunked_prefill"] = bench_chunked(impl, dist, stepper, K, Wm, peaks, traffic)
        if impl.kind == "nc":
            extra["decode_step_gemms"] = bench_gemm(dist, stepper, K, Wm, peaks, traffic)
            extra["prompt_pass_gemms"] = bench_prompt_gemm(dist, stepper, K, Wm, peaks)
            extra["cfg5_e2e_generation"] = bench_cfg5(dist)
        else:
            extra["cfg5_e2e_generation"] = bench_cfg5_reference(dist)
    clk = clocks.stop()

    line = {
        "metric": "prefill attn TFLOP/s @2048 causal",
        "value": head["value"],
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": K,
        "warmup": Wm,
        "ms_per_step": head["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V at the BASELINE shapes)",
        "config": {
            "workload": "cfg2: causal prefill, 1 sequence x 2048 positions per GPU, 17 heads x 128;"
                        " step = fused RoPE+QK-norm+KV-append pass + prefill attention",
            "seq_len": W.CFG2_SEQ, "heads": H, "head_dim": D, "sequences_per_gpu": 1,
            "l2": f"inputs larger than L2: steps rotate over {head['input_sets']} independent input "
                  "sets (> 2x L2 together), so each step starts with its inputs out of L2",
            "timing": "K steps back to back between two CUDA events on the launching stream, behind a "
                      "GPU-side hold spin covering the host's launches (e2e counts host cost)",
            "parallelism": f"replica x{args.gpus} (independent sequences, no collective)",
        },
        "attn_kernel_ms": head["attn_kernel_ms"],
        "prologue_ms": head["prologue_ms"],
        "roofline": head["roofline"],
        "e2e": head["e2e"],
        "gpu_launches": head["gpu_launches"],
        "clocks": clk,
        "extra": extra,
    }
    if args.impl == "reference":
        line["impl"] = "reference"
        line["gpu_launches"] = 0
        line["reference_kind"] = ("the reference's own CUDA kernels (kernels/rope.cu, "
                                  "kernels/flash_attention.cu) rebuilt for sm_100a, called in "
                                  "the reference's order; the reference has no CPU path")
        line["cpu_baseline"] = {"value": head["value"], "unit": "TFLOP/s", "cores": 0,
                                "kind": "reference",
                                "sample": "full cfg2 on one B200 through the reference kernels"}
    elif dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline_prefill()
    if impl.kind == "nc":
        st = impl.nc.device_status(reset=True)
        line["device_status"] = st
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()

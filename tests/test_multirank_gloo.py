"""Multi-process logic of bench.py on CPU (gloo, world size 2): the sequence sharding that
replaces any data-path collective, the max/sum reductions of per-rank results, and failure
detection when one rank dies (host-side fault only, no GPU involved)."""
import os
import socket
import subprocess
import sys
import textwrap

import pytest

from conftest import ROOT


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(body, world=2, timeout=120):
    port = free_port()
    script = textwrap.dedent(f"""
        import os, sys, json
        sys.path.insert(0, {ROOT!r})
        import bench
        from nanochat_inferonly_lightning_b200 import workloads as W
        rank = int(os.environ["RANK"])
    """) + textwrap.dedent(body)
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(world),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, "-c", script], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            o, e = p.communicate()
        outs.append((p.returncode, o, e))
    return outs


def test_shards_cover_every_sequence_once():
    for n in (1, 2, 3, 4, 8, 64):
        for world in (1, 2, 4, 8):
            spans = [__import__("nanochat_inferonly_lightning_b200.workloads",
                                fromlist=["shard"]).shard(n, r, world) for r in range(world)]
            covered = [i for a, b in spans for i in range(a, b)]
            assert covered == list(range(n))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_weighted_shards_cover_every_sequence_once_and_balance_bytes():
    """The decode benches cut the sequences into contiguous shares of about equal KV length:
    every sequence once, in order, at least one per rank when there are enough, and each
    rank's sum within one sequence's length of an equal share."""
    from nanochat_inferonly_lightning_b200 import workloads as W

    cases = [W.cfg3_kv_lens(), [512], [5, 1, 1, 1], [7] * 9, list(range(1, 40))]
    for lens in cases:
        for world in (1, 2, 4, 8):
            spans = [W.shard_weighted(lens, r, world) for r in range(world)]
            covered = [i for a, b in spans for i in range(a, b)]
            assert covered == list(range(len(lens)))
            if len(lens) >= world:
                assert all(b > a for a, b in spans)
                share = sum(lens) / world
                assert all(abs(sum(lens[a:b]) - share) <= max(lens) * (1 + 1e-9)
                           for a, b in spans), (lens, world, spans)
    assert W.shard_weighted([512], 0, 2) == (0, 1)


def test_two_ranks_shard_and_reduce():
    outs = run_ranks("""
        d = bench.Dist(2, backend="gloo", timeout_s=30)
        lens = W.cfg3_kv_lens()
        a, b = W.shard(len(lens), d.rank, d.world)
        mine = W.decode_bytes(lens[a:b])
        total = d.sum(mine)
        slowest = d.max(1.0 + d.rank)
        d.barrier()
        print(json.dumps({"rank": d.rank, "span": [a, b], "total": total, "max": slowest}))
        d.close()
    """)
    for rc, o, e in outs:
        assert rc == 0, e
    res = [__import__("json").loads(o.strip().splitlines()[-1]) for _, o, _ in outs]
    from nanochat_inferonly_lightning_b200 import workloads as W

    assert res[0]["span"] == [0, 32] and res[1]["span"] == [32, 64]
    assert all(r["total"] == W.cfg3_bytes() for r in res)
    assert all(r["max"] == 2.0 for r in res)


def test_dead_rank_is_reported_not_hung():
    """Rank 1 raises before the first collective; rank 0's reduction must end with an error
    (process-group timeout or peer-closed connection) instead of waiting forever, and the
    launcher sees both failures."""
    outs = run_ranks("""
        d = bench.Dist(2, backend="gloo", timeout_s=10)
        if d.rank == 1:
            raise RuntimeError("injected failure on rank 1")
        try:
            d.max(1.0)
            print("UNEXPECTED: reduction completed")
            sys.exit(0)
        except Exception as exc:
            print("rank0 saw:", type(exc).__name__)
            sys.exit(3)
    """, timeout=90)
    (rc0, o0, e0), (rc1, o1, e1) = outs
    assert rc1 != 0 and "injected failure" in e1
    assert rc0 == 3, (o0, e0)

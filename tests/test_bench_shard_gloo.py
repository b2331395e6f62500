"""The multi-GPU split of bench.py's workload, on two CPU ranks over gloo.

bench.py divides the FIXED workload into contiguous (batch, head) slice
ranges, one per rank, each rank drawing the whole config from BASELINE's
generator and cutting out its slices.  Here each gloo rank runs its range
through the oracle (the GPU kernels' stand-in), the ranks' outputs are
gathered, and the whole must equal one run over all slices; the step time is
reduced with MAX as bench.py does.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

CFG = (5, 96, 80, 32, True, 7, 0.5, "test")


def _worker(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O
        bh, sq, sk, d, causal = CFG[:5]
        h0, h1 = bench.shard_range(bh, world, rank)
        q, k, v = bench.seeded_inputs(CFG, h0, h1)
        out, lse, _ = O.flash_v2_multihead(q, k, v, h1 - h0, sq, sk, d, causal, nthreads=1)
        # pad to the largest range so all_gather has equal sizes
        per = -(-bh // world)
        o = torch.zeros(per * sq * d)
        o[: out.size] = torch.from_numpy(out)
        gathered = [torch.zeros_like(o) for _ in range(world)]
        dist.all_gather(gathered, o)
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            parts = []
            for r in range(world):
                a, b = bench.shard_range(bh, world, r)
                parts.append(gathered[r].numpy()[: (b - a) * sq * d])
            ret["out"] = np.concatenate(parts)
            ret["tmax"] = float(t.item())
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_ranges_partition_the_slices():
    for bh in (1, 5, 32, 256):
        for world in (1, 2, 3, 8):
            got = [bench.shard_range(bh, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == bh
            assert all(got[i][1] == got[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in got) - min(b - a for a, b in got) <= 1


def test_seeded_slices_equal_the_whole_draw():
    q, k, v = bench.seeded_inputs(CFG)
    q2, k2, v2 = bench.seeded_inputs(CFG, 2, 4)
    bh, sq, sk, d = CFG[:4]
    assert np.array_equal(q2, q[2 * sq * d:4 * sq * d])
    assert np.array_equal(v2, v[2 * sk * d:4 * sk * d])
    # BASELINE's generator: default_rng(seed), Q then K then V, times the factor
    rng = np.random.default_rng(CFG[5])
    assert np.array_equal(q, rng.standard_normal(bh * sq * d, dtype=np.float32) * np.float32(0.5))


def test_two_gloo_ranks_cover_the_fixed_workload():
    import oracle as O
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    ret = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    bh, sq, sk, d, causal = CFG[:5]
    q, k, v = bench.seeded_inputs(CFG)
    want, _, _ = O.flash_v2_multihead(q, k, v, bh, sq, sk, d, causal, nthreads=1)
    assert np.array_equal(ret["out"], want)
    assert ret["tmax"] == 2.0

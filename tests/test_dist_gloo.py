"""Data-parallel bookkeeping of bench.py on two CPU ranks (gloo): every rank gets its own
sequences (disjoint prompt seeds, deterministic per rank) and timings reduce to the max."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = dict(bench.WORKLOADS["depth12_bs1"], B=3, prompt=8)
        pr, rng = bench.prompts_for(w, rank)
        mine = torch.tensor(pr.astype("int64"))
        allp = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allp, mine)
        t = bench.allmax(dist, float(rank + 1.5))
        q.put((rank, [a.tolist() for a in allp], t, int(rng[0])))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_ranks_disjoint_sequences_and_max_timing():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=100) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    res.sort()
    (r0, g0, t0, s0), (r1, g1, t1, s1) = res
    assert g0 == g1                       # everyone sees the same gathered prompts
    assert g0[0] != g0[1]                 # ranks decode different sequences
    assert t0 == t1 == 2.5                # timing is the max over ranks
    assert s0 != s1

"""The N > 1 host path on CPU with gloo ranks (world size 2, 127.0.0.1): row sharding + loss-sum all-reduce equal
the unsharded result, and a rank that leaves early makes its peer's collective fail within the timeout instead of
hanging (failure made on the host; no GPU involved)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from sdmchat_b200.dist import shard_rows


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_partition():
    for total in (1, 7, 32, 33):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _loss_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from goldens import load, lm_params
    from oracle import sdm_oracle as O
    from sdmchat_b200 import dist as D
    D.init("gloo", timeout_s=30)
    g = load("lm_full")
    P = lm_params(g)
    idx = g["idx"]
    lo, hi = D.shard_rows(idx.shape[0], rank, world)
    lg = O.lm_forward(P, idx[lo:hi], bf16_stream=True, chunk=16, margins=False)
    part = O.ce_sum(lg[:, :-1], idx[lo:hi, 1:])
    tot, cnt = D.reduce_loss(part, (hi - lo) * (idx.shape[1] - 1))
    # bench.py's per-step exchange: the in-place all-reduce of (loss sum, token count), then the slowest rank's time
    import torch
    buf = torch.tensor([part, float((hi - lo) * (idx.shape[1] - 1))], dtype=torch.float64)
    D.all_reduce_(buf)
    slowest = D.max_over_ranks(1.0 + rank)
    D.barrier()
    q.put((rank, tot, cnt, float(buf[0]), float(buf[1]), slowest, D.world_size()))
    D.finalize()


def test_sharded_loss_sum_equals_unsharded():
    from goldens import load, lm_params
    from oracle import sdm_oracle as O
    g = load("lm_full")
    lg = O.lm_forward(lm_params(g), g["idx"], bf16_stream=True, chunk=16, margins=False)
    want = O.ce_sum(lg[:, :-1], g["idx"][:, 1:])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_loss_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for _, tot, cnt, tot2, cnt2, slowest, world in res:
        assert cnt == cnt2 == g["idx"].shape[0] * (g["idx"].shape[1] - 1)
        assert abs(tot - want) / abs(want) < 1e-6 and abs(tot2 - want) / abs(want) < 1e-6
        assert slowest == 2.0 and world == 2


def _early_exit_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch
    import torch.distributed as dist
    from sdmchat_b200 import dist as D
    D.init("gloo", timeout_s=5)
    dist.barrier()
    def report(msg):
        q.put((rank, msg))
        q.close()
        q.join_thread()  # flush the queue's feeder thread before the hard exit

    if rank == 1:
        report("left")
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        D.reduce_loss(torch.tensor(1.0), 1)
        report("no error")
    except Exception as e:  # the peer is gone: the all-reduce must fail, not hang
        report("error:" + type(e).__name__)
    os._exit(0)


def test_rank_leaving_early_fails_peer_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_early_exit_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error:"), res[0]

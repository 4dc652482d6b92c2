"""Failure detection on the host: a rank that leaves a sharded run between
steps is noticed by the others at their next collective, which ends with an
error within the process group's timeout instead of hanging.  Run as three
gloo ranks on CPU through the layer's own mate-frame exchange
(multics_b200.sharded.exchange_mate_frames)."""

import os
import time

import numpy as np
import pytest
import torch

from test_sharded_cpu import _regrouped_labels

TIMEOUT_S = 5.0


def _rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    from multics_b200.sharded import ShardTopology, exchange_mate_frames

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))
    P, T, L, N, KL, KG, dim = 8, 6, 3, 4, 2, 2, 4
    lab = _regrouped_labels(P, T, 3, seed=7)
    S = P * T * L + T * (N * KL + KG)
    k_all = torch.arange(S * dim, dtype=torch.float32).reshape(S, dim)
    t = ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=1, local_attn=-1,
                      direct=True, labels=lab, world=world, rank=rank)
    loc = torch.from_numpy(t.local_rows())
    k, v = k_all[loc], -k_all[loc]
    remote = torch.zeros((max(sum(t.recv_units) * L, 1), 2 * dim))
    exchange_mate_frames(t, k, v, remote)  # step 1: every rank takes part
    dist.barrier()
    if rank == world - 1:
        q.put((rank, "left", 0.0))
        os._exit(0)  # leaves between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        exchange_mate_frames(t, k, v, remote)  # step 2: one rank is gone
        dist.barrier()
        q.put((rank, "no error", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - the point is that it raises
        q.put((rank, type(e).__name__, time.monotonic() - t0))
    os._exit(0)


def test_departed_rank_is_detected_by_the_others():
    import torch.multiprocessing as mp

    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = 29800 + os.getpid() % 150
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = sorted(q.get() for _ in range(world))
    assert res[-1][:2] == (world - 1, "left")
    for rank, outcome, waited in res[:-1]:
        assert outcome != "no error", (rank, outcome)
        assert waited < 3 * TIMEOUT_S + 5, (rank, waited)

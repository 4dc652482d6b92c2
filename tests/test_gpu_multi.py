"""Player-sharded layer over NCCL: one process per GPU (every GPU of the
box, 2 to 8), group-mate
frames by all_to_all or read in place from the peer's memory, hub rows merged
by log-sum-exp over the ranks' partial rows (all-gathered, or read in place
from the peers), checked against the oracle.  Skipped on boxes with fewer
than two GPUs.  NVLink multicast is switched off in NCCL and in torch's
symmetric memory: the test needs only plain peer pointers."""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = max(2, min(torch.cuda.device_count() if torch.cuda.is_available() else 0, 8))


def _rank_main(rank, world, port, q, transport):
    import datetime

    import torch.distributed as dist

    from oracle import hier_oracle as O
    from multics_b200.sharded import ShardedHierAttention, ShardTopology
    from test_sharded_cpu import _regrouped_labels

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        P, T, L, N, KL, KG, H = 8, 6, 40, 4, 4, 3, 2
        lab = _regrouped_labels(P, T, 3, seed=3)
        S = P * T * L + T * (N * KL + KG)
        g = torch.Generator().manual_seed(1)
        mk = lambda: (torch.randn((S, H * 128), generator=g) * 0.5).to(torch.bfloat16)  # noqa: E731
        qa, ka, va = mk(), mk(), mk()
        t = ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=1, local_attn=-1,
                          direct=True, labels=lab, world=world, rank=rank)
        loc = torch.from_numpy(t.local_rows())
        dev = torch.device("cuda", rank)
        ql, kl, vl = (x[loc].contiguous().to(dev) for x in (qa, ka, va))
        sh = ShardedHierAttention(t, H, dev, transport=transport)
        out = sh.forward(ql, kl, vl)
        out2 = sh.forward(ql, kl, vl)  # a second step over the same buffers
        assert torch.equal(out, out2)
        torch.cuda.synchronize(dev)
        sh.check_status()
        act = O.active_from_labels(lab, N)
        dense = O.dense_mask(P, T, L, N, KL, KG, 1, -1, labels=lab, active=act, direct=True)
        f = lambda x: x.float().numpy()  # noqa: E731
        rows = t.local_rows()
        ref = O.masked_attention(f(qa)[rows], f(ka), f(va), H, lambda r0, r1: dense[rows[r0:r1]])
        o = out.float().cpu().numpy()
        err = float(np.abs(o - ref).max())
        cos = float((o * ref).sum() / (np.linalg.norm(o) * np.linalg.norm(ref)))
        q.put((rank, err, cos, len(t.needs[rank])))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs two GPUs")
@pytest.mark.parametrize("transport", ["exchange", "peer"])
def test_sharded_layer_over_nccl(transport):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = 29700 + os.getpid() % 200
    port += 1 if transport == "peer" else 0
    procs = [ctx.Process(target=_rank_main, args=(r, WORLD, port, q, transport))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get() for _ in range(WORLD))
    for rank, err, cos, n_units in res:
        assert err <= 2e-2, (rank, err)
        assert cos >= 0.9995, (rank, cos)
        assert n_units > 0

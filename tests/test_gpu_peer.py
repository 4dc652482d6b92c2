"""Peer reads over NVLink, in one process driving two GPUs.

The sharded layer's peer transport lets the attention kernel read the other
ranks' key/value rows in place (plain TMA loads of peer memory, no
multicast).  Here rank 0 of a two-rank topology runs its own peer-transport
plan on GPU 0 with rank 1's rows on GPU 1 (peer access enabled), and again
with a copy of those rows on GPU 0: the outputs are bitwise equal, and the
player rows rank 0 computes match the oracle's fp32 attention.  The test
prints the key/value bytes its plan requests from the peer (the expected
NVLink payload of the first launch).  It needs two GPUs with peer access
and skips otherwise.
"""

import json

import numpy as np
import pytest
import torch

from oracle import hier_oracle as O
from test_sharded_cpu import _regrouped_labels

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


def _enable_peer_access(dev, peer):
    """Peer access from ``dev`` to ``peer``'s memory; False when unavailable."""
    if torch.cuda.device_count() <= max(dev, peer):
        return False
    if not torch.cuda.can_device_access_peer(dev, peer):
        return False
    from cuda.bindings import runtime as cudart

    torch.cuda.set_device(dev)
    torch.zeros(1, device=f"cuda:{dev}")  # the primary context exists
    (err,) = cudart.cudaDeviceEnablePeerAccess(peer, 0)
    return err in (cudart.cudaError_t.cudaSuccess,
                   cudart.cudaError_t.cudaErrorPeerAccessAlreadyEnabled)


class _DeviceRows:
    """Rows of a bf16 [rows, cols] buffer from cudaMalloc on ``dev`` (memory
    that peer access enabled by cudaDeviceEnablePeerAccess covers), with what
    the stream table reads of a tensor: data_ptr(), shape, stride()."""

    def __init__(self, host, dev):
        from cuda.bindings import runtime as cudart

        host = host.contiguous()
        self.shape = tuple(host.shape)
        n = host.numel() * host.element_size()
        (err,) = cudart.cudaSetDevice(dev)
        assert err == cudart.cudaError_t.cudaSuccess
        err, self.ptr = cudart.cudaMalloc(n)
        assert err == cudart.cudaError_t.cudaSuccess
        (err,) = cudart.cudaMemcpy(self.ptr, host.data_ptr(), n,
                                   cudart.cudaMemcpyKind.cudaMemcpyHostToDevice)
        assert err == cudart.cudaError_t.cudaSuccess
        (err,) = cudart.cudaSetDevice(0)
        assert err == cudart.cudaError_t.cudaSuccess

    def data_ptr(self):
        return int(self.ptr)

    def stride(self, i):
        return (self.shape[1], 1)[i]

    def free(self):
        from cuda.bindings import runtime as cudart

        cudart.cudaFree(self.ptr)


def test_peer_rows_on_second_gpu_match_local_copy(monkeypatch):
    if not _enable_peer_access(0, 1):
        pytest.skip("needs two GPUs with peer access")
    from multics_b200.sharded import ShardedHierAttention, ShardTopology

    P, T, L, N, KL, KG, H = 8, 6, 40, 4, 4, 3, 2
    lab = _regrouped_labels(P, T, 3, seed=3)
    S = P * T * L + T * (N * KL + KG)
    g = torch.Generator().manual_seed(7)
    q, k, v = ((torch.randn((S, H * 128), generator=g) * 0.5).to(torch.bfloat16)
               for _ in range(3))
    d0 = torch.device("cuda:0")
    topo = [ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=1, local_attn=-1,
                          direct=True, labels=lab, world=2, rank=r) for r in range(2)]
    # rank 0's peer-transport plan; the process-group setup (symmetric memory,
    # rendezvous) is replaced by buffers this process owns
    monkeypatch.setattr(ShardedHierAttention, "_setup_peer", lambda self: None)
    sh = ShardedHierAttention(topo[0], H, d0, transport="peer", spread_hub_keys=False)
    assert sh.transport == "peer"
    t0 = topo[0]
    rows = max(len(x) for x in t0.local) * T * L + t0.hub_rows
    sh._sym = torch.zeros((2, rows, H * 128), dtype=torch.bfloat16, device=d0)
    loc0 = torch.from_numpy(t0.local_rows())
    ql = q[loc0].to(d0)
    sh.k_buffer().copy_(k[loc0])
    sh.v_buffer().copy_(v[loc0])
    n1 = len(t0.local[1]) * T * L  # rank 1's player rows, in its local order
    loc1 = torch.from_numpy(topo[1].local_rows()[:n1])
    k1, v1 = _DeviceRows(k[loc1], 1), _DeviceRows(v[loc1], 1)

    # key/value boxes the plan reads from stream 2 and up (the peer's rows)
    qp = sh.q_pairs[:sh.n_pairs].cpu().numpy()
    kv = sh.kv_tiles.cpu().numpy()
    boxes = sum(int(((kv[qp[p, 4]:qp[p, 5], :2] >> 24) >= 2).sum()) for p in range(sh.n_pairs))
    assert boxes > 0, "the plan reads no peer rows"

    outs, parts = [], []
    for peer in ((k1, v1), (k[loc1].to(d0), v[loc1].to(d0))):
        sh._peers = [peer]
        o = torch.zeros_like(ql)
        sh.part_o.zero_()
        sh.attend(ql, sh.k_buffer(), sh.v_buffer(), o)
        torch.cuda.synchronize(d0)
        sh.check_status()
        assert int(sh.err.item()) == 0
        outs.append(o.clone())
        parts.append(sh.part_o.clone())
    k1.free()
    v1.free()
    assert torch.equal(outs[0], outs[1]), "peer reads differ from local reads"
    assert torch.equal(parts[0], parts[1])
    print(json.dumps({"peer_boxes": boxes, "heads": H,
                      "peer_kv_bytes_requested": boxes * H * 2 * 64 * 128 * 2}))

    # the player rows rank 0 computes are final: check them against the oracle
    act = O.active_from_labels(lab, N)
    dense = O.dense_mask(P, T, L, N, KL, KG, 1, -1, labels=lab, active=act, direct=True)
    f = lambda t: t.float().numpy()  # noqa: E731
    ref = O.masked_attention(f(q), f(k), f(v), H, lambda r0, r1: dense[r0:r1])
    mine = t0.computed_rows()
    got = outs[0].float().cpu().numpy()[mine]
    want = ref[loc0.numpy()[mine]]
    err = np.abs(got - want).max()
    cos = (got * want).sum() / (np.linalg.norm(got) * np.linalg.norm(want))
    assert err <= MAX_ABS, err
    assert cos >= MIN_COS, cos

"""Player-sharded layer on one GPU: every rank's plan, attention launch and
the hub merge run in one process (the exchange copies the mate frames, the
merge sums the partials), and the assembled output is compared with the
oracle's dense-mask fp32 attention.  The NCCL version runs in
test_gpu_multi.py when a box has two GPUs."""

import numpy as np
import pytest
import torch

from oracle import hier_oracle as O
from test_sharded_cpu import _regrouped_labels

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


def _case(P, T, L, N, KL, KG, labels, H, seed, n_block=1, win=-1):
    S = P * T * L + T * (N * KL + KG)
    g = torch.Generator().manual_seed(seed)
    mk = lambda: (torch.randn((S, H * 128), generator=g) * 0.5).to(torch.bfloat16)  # noqa: E731
    q, k, v = mk(), mk(), mk()
    act = O.active_from_labels(labels, N)
    dense = O.dense_mask(P, T, L, N, KL, KG, n_block, win, labels=labels, active=act,
                         direct=True)
    f = lambda t: t.float().numpy()  # noqa: E731
    ref = O.masked_attention(f(q), f(k), f(v), H, lambda r0, r1: dense[r0:r1])
    return q, k, v, ref


def _run_sharded(P, T, L, N, KL, KG, labels, H, world, q, k, v, n_block=1, win=-1,
                 spread=False):
    """Every rank's plan and attention launch in one process; the ranks'
    player-partial slots are copied together as the all-gather would, then
    merged.  With ``spread`` the ranks share the hub-token partial pairs and
    the merge reads every partial from its rank's buffer, as the peer
    transport's merge does (all buffers are on this GPU)."""
    import ctypes

    from multics_b200 import _lib
    from multics_b200._lib import check, ptr, stream_ptr
    from multics_b200.sharded import ShardedHierAttention, ShardTopology

    S = q.shape[0]
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = torch.zeros((S, H * 128), dtype=torch.float32, device="cuda")
    shards = []
    for rank in range(world):
        t = ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=n_block, local_attn=win,
                          direct=True, labels=labels, world=world, rank=rank)
        sh = ShardedHierAttention(t, H, "cuda", spread_hub_keys=spread)
        loc = torch.from_numpy(t.local_rows()).cuda()
        ql, kl, vl = qc[loc].contiguous(), kc[loc].contiguous(), vc[loc].contiguous()
        sh.fill_remote_from(kc, vc)
        o = torch.empty_like(ql)
        sh.attend(ql, kl, vl, o)
        sh.check_status()
        mine = torch.from_numpy(t.computed_rows()).cuda()
        out[loc[mine]] = o[mine].float()
        shards.append(sh)
    s0 = shards[0]
    h0, slot = s0.topo.hub_rows, s0.topo.hub_partial_slot
    if spread and world > 1:
        dev = torch.device("cuda")
        ob = torch.tensor([sh.part_o.data_ptr() for sh in shards], dtype=torch.int64, device=dev)
        lb = torch.tensor([sh.part_lse.data_ptr() for sh in shards], dtype=torch.int64,
                          device=dev)
        merged = torch.empty((h0, H * 128), dtype=torch.bfloat16, device=dev)
        check(_lib.lib().hier_lse_gather_merge_peers(
            ptr(ob), ptr(lb), world, 0, h0, max(slot, 1), s0.part_o.stride(0), H, 128,
            ptr(s0.csr_off), ptr(s0.csr_rows), h0, ptr(merged), merged.stride(0), None,
            ptr(s0.hub_key_owner), stream_ptr(dev)))
        out[torch.from_numpy(s0.topo.hub_rows_order()).cuda()] = merged.float()
        return out.cpu().numpy()
    # the all-gather: every rank's player-partial slot into rank 0's buffer
    for r, sh in enumerate(shards[1:], start=1):
        rows = slice(h0 + r * slot, h0 + (r + 1) * slot)
        s0.part_o[rows] = sh.part_o[rows]
        s0.part_lse[rows] = sh.part_lse[rows]
    merged = torch.empty((h0, H * 128), dtype=torch.bfloat16, device="cuda")
    s0.merge_partials(merged)
    out[torch.from_numpy(s0.topo.hub_rows_order()).cuda()] = merged.float()
    return out.cpu().numpy()


def _check(o, ref):
    assert np.isfinite(o).all()
    err = np.abs(o - ref).max()
    cos = (o * ref).sum() / (np.linalg.norm(o) * np.linalg.norm(ref))
    assert err <= MAX_ABS, err
    assert cos >= MIN_COS, cos


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_sharded_dynamic_groups_match_oracle(world):
    """Config-4 shape in miniature: 8 players, 4 groups of 2 regrouped every
    3 frames (mates move between ranks)."""
    P, T, L, N, KL, KG, H = 8, 6, 40, 4, 4, 3, 2
    lab = _regrouped_labels(P, T, 3, seed=3)
    q, k, v, ref = _case(P, T, L, N, KL, KG, lab, H, seed=1)
    _check(_run_sharded(P, T, L, N, KL, KG, lab, H, world, q, k, v), ref)


@pytest.mark.parametrize("world", [3, 4, 8])
def test_sharded_uneven_players_match_oracle(world):
    """Config-5 grouping in miniature: 10 players in groups (3,3,2,2), split
    between the ranks by 256-row strips (players shared by two ranks)."""
    P, T, L, N, KL, KG, H = 10, 4, 24, 4, 3, 2, 2
    lab = np.array([[0, 0, 0, 1, 1, 1, 2, 2, 3, 3]] * T)
    q, k, v, ref = _case(P, T, L, N, KL, KG, lab, H, seed=2)
    _check(_run_sharded(P, T, L, N, KL, KG, lab, H, world, q, k, v), ref)


@pytest.mark.parametrize("world", [1, 2])
def test_sharded_inactive_groups_match_oracle(world):
    """Frames where a group has no member: its hub rows attend to themselves
    only (the mask's inactive-local self edge), and no player reaches them."""
    P, T, L, N, KL, KG, H = 4, 6, 36, 3, 5, 2, 2
    lab = np.array([[0, 0, 1, 1]] * 3 + [[0, 2, 2, 0]] * 3)  # group 2 idle, then group 1
    q, k, v, ref = _case(P, T, L, N, KL, KG, lab, H, seed=4)
    _check(_run_sharded(P, T, L, N, KL, KG, lab, H, world, q, k, v), ref)


@pytest.mark.parametrize("world", [1, 2])
def test_sharded_blocks_and_window_match_oracle(world):
    """Temporal blocks of 3 frames with a 3-frame window, groups reassigned
    per block; 20 frames of local hubs (more than one 128-row hub tile per
    group)."""
    P, T, L, N, KL, KG, H = 4, 12, 24, 2, 16, 6, 2
    lab = _regrouped_labels(P, T, 3, seed=5)
    q, k, v, ref = _case(P, T, L, N, KL, KG, lab, H, seed=5, n_block=3, win=3)
    _check(_run_sharded(P, T, L, N, KL, KG, lab, H, world, q, k, v, n_block=3, win=3), ref)


@pytest.mark.parametrize("world", [3, 5])
def test_sharded_strip_split_dynamic_groups_match_oracle(world):
    """Players split between ranks by strips while groups change every 3
    frames: mate frames come from the players' home ranks."""
    P, T, L, N, KL, KG, H = 8, 6, 100, 4, 4, 3, 2
    lab = _regrouped_labels(P, T, 3, seed=9)
    q, k, v, ref = _case(P, T, L, N, KL, KG, lab, H, seed=9)
    _check(_run_sharded(P, T, L, N, KL, KG, lab, H, world, q, k, v), ref)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_spread_hub_keys_match_oracle(world):
    """The hub-token partial pairs shared out among the ranks (the peer
    transport's default) and each hub row merged from the partials on their
    ranks: dynamic groups, and enough hub frames for several hub-key pairs per
    group."""
    P, T, L, N, KL, KG, H = 8, 6, 40, 4, 4, 3, 2
    lab = _regrouped_labels(P, T, 3, seed=3)
    q, k, v, ref = _case(P, T, L, N, KL, KG, lab, H, seed=1)
    _check(_run_sharded(P, T, L, N, KL, KG, lab, H, world, q, k, v, spread=True), ref)
    P, T, L, N, KL, KG = 4, 20, 24, 2, 16, 6
    lab = _regrouped_labels(P, T, 4, seed=6)
    q, k, v, ref = _case(P, T, L, N, KL, KG, lab, H, seed=6, n_block=2, win=5)
    _check(_run_sharded(P, T, L, N, KL, KG, lab, H, min(world, 4), q, k, v, n_block=2, win=5,
                        spread=True), ref)

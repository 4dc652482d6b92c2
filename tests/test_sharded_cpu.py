"""Host logic of the player-sharded layer on CPU: player split, the remote
units each rank's direct edges need (checked against the dense mask), and
the all_to_all exchange order with two gloo ranks."""

import os

import numpy as np
import pytest
import torch

from oracle import hier_oracle as O


def _regrouped_labels(P, T, every, seed, group_size=2):
    rng = np.random.default_rng(seed)
    lab = np.zeros((T, P), np.int64)
    for t0 in range(0, T, every):
        perm = rng.permutation(P)
        row = np.empty(P, np.int64)
        row[perm] = np.arange(P) // group_size
        lab[t0:t0 + every] = row
    return lab


def test_split_players():
    from multics_b200.sharded import split_players

    assert split_players(8, 8) == [(i, i + 1) for i in range(8)]
    assert split_players(10, 8) == [(0, 2), (2, 4), (4, 5), (5, 6), (6, 7), (7, 8), (8, 9), (9, 10)]
    assert split_players(4, 1) == [(0, 4)]
    with pytest.raises(ValueError):
        split_players(2, 3)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("n_block", [1, 3])
def test_remote_units_match_dense_mask(world, n_block):
    from multics_b200.sharded import ShardTopology

    P, T, L, N, KL, KG = 8, 6, 2, 4, 2, 2
    lab = _regrouped_labels(P, T, 3, seed=world)
    act = O.active_from_labels(lab, N)
    dense = O.dense_mask(P, T, L, N, KL, KG, n_block, -1, labels=lab, active=act, direct=True)
    for rank in range(world):
        t = ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=n_block, local_attn=-1,
                          direct=True, labels=lab, world=world, rank=rank)
        rows = np.concatenate([p * T * L + np.arange(b * 256, min(e * 256, T * L))
                               for p, b, e in t.segments[rank]])
        cols = np.nonzero(dense[rows].any(0))[0]
        want = set()
        for c in cols:
            if c < P * T * L:
                o, f = c // (T * L), (c % (T * L)) // L
                if o not in t.local_players:
                    want.add((o, f))
        assert set(t.needs[rank]) == want
        # every entry of the exchange table points at its own slot
        keys = t.remote_keys("exchange")
        for i, (o, f) in enumerate(t.needs[rank]):
            assert keys[o * T + f] == (2 << 24) | (i * L)


def test_static_groups_on_one_rank_exchange_nothing():
    from multics_b200.sharded import ShardTopology

    lab = np.array([[0, 0, 1, 1]] * 4)
    t = ShardTopology(P=4, T=4, L=3, N=2, KL=2, KG=1, n_block=1, local_attn=-1, direct=True,
                      labels=lab, world=2, rank=0)
    assert t.needs == [[], []] and t.send_rows.size == 0


def _exchange_rank(rank, world, port, q):
    import torch.distributed as dist

    from multics_b200.sharded import ShardTopology, exchange_mate_frames

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P, T, L, N, KL, KG, dim = 8, 6, 3, 4, 2, 2, 4
        lab = _regrouped_labels(P, T, 3, seed=7)
        S = P * T * L + T * (N * KL + KG)
        k_all = torch.arange(S * dim, dtype=torch.float32).reshape(S, dim)
        v_all = -k_all
        t = ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=1, local_attn=-1,
                          direct=True, labels=lab, world=world, rank=rank)
        loc = torch.from_numpy(t.local_rows())
        k, v = k_all[loc], v_all[loc]
        n = sum(t.recv_units) * L
        remote = torch.full((max(n, 1), 2 * dim), float("nan"))
        exchange_mate_frames(t, k, v, remote)
        ok = True
        for i, (o, f) in enumerate(t.needs[rank]):
            src = (o * T + f) * L
            ok &= torch.equal(remote[i * L:(i + 1) * L, :dim], k_all[src:src + L])
            ok &= torch.equal(remote[i * L:(i + 1) * L, dim:], v_all[src:src + L])
        q.put((rank, bool(ok), len(t.needs[rank])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_with_gloo_ranks(world):
    """All-to-all of the mate frames with whole players per rank (2 ranks)
    and with players split between ranks by strips (3 ranks)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = 29600 + os.getpid() % 200 + world
    procs = [ctx.Process(target=_exchange_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = sorted(q.get() for _ in range(world))
    assert all(p.exitcode == 0 for p in procs)
    assert all(r[1] for r in res)
    assert all(r[2] > 0 for r in res)  # dynamic groups do cross ranks


def test_local_rows_hubs_group_major():
    from multics_b200.sharded import ShardTopology

    P, T, L, N, KL, KG = 4, 3, 5, 2, 2, 1
    lab = np.array([[0, 0, 1, 1]] * T)
    t = ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=1, local_attn=-1, direct=True,
                      labels=lab, world=2, rank=1)
    rows = t.local_rows()
    A = P * T * L
    assert list(rows[:t.own_rows]) == list(range(2 * T * L, 4 * T * L))
    hub = rows[t.own_rows:] - A
    assert sorted(hub) == list(range(T * (N * KL + KG)))
    # group 0 frames 0..2, then group 1 frames 0..2 (slots inside), then globals
    f_major = lambda f, g, s: (f * N + g) * KL + s  # noqa: E731
    expect = [f_major(f, g, s) for g in range(N) for f in range(T) for s in range(KL)]
    expect += list(range(T * N * KL, T * (N * KL + KG)))
    assert list(hub) == expect


@pytest.mark.parametrize("P,T,L,world,KL", [(8, 6, 3, 2, 2), (8, 42, 220, 8, 16),
                                            (10, 42, 220, 8, 16), (10, 42, 220, 4, 16),
                                            (5, 6, 40, 3, 0), (4, 3, 16, 1, 8)])
def test_split_strips_covers_and_balances(P, T, L, world, KL):
    """Every strip of every player on exactly one rank, contiguous runs per
    rank, whole players when the ranks divide the players, work (hub
    partials counted on the home rank) within two strips of equal."""
    from multics_b200.sharded import split_strips, strip_weights

    nps = -(-T * L // 256)
    segs = split_strips(P, T, L, world, KL)
    seen = np.zeros((P, nps), np.int64)
    w = strip_weights(T, L, KL)
    loads = []
    for r in range(world):
        load = 0.0
        for p, b, e in segs[r]:
            seen[p, b:e] += 1
            load += w[b:e].sum()
        loads.append(load)
    assert (seen == 1).all()
    if P % world == 0:
        per = P // world
        assert all([p for p, _, _ in segs[r]] == list(range(r * per, (r + 1) * per))
                   and all(b == 0 and e == nps for _, b, e in segs[r]) for r in range(world))
    assert max(loads) - min(loads) <= 2 * w.max() + 1e-9


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_hub_partials_cover_each_hub_row_once_per_key_set(world):
    """In the assembled partial-row buffer every local hub row has its
    hub-token partial and one partial per member player, in the slot of the
    rank that owns the player; global hub rows only the hub-token one."""
    from multics_b200.sharded import ShardTopology

    P, T, L, N, KL, KG = 8, 6, 3, 4, 2, 3
    lab = _regrouped_labels(P, T, 3, seed=7)
    tops = [ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=1, local_attn=-1,
                          direct=True, labels=lab, world=world, rank=r) for r in range(world)]
    t = tops[0]
    off, rows = t.hub_partials()
    assert all((x.hub_partials()[1] == rows).all() for x in tops)  # the same on every rank
    slot = t.hub_partial_slot
    for r in range(t.hub_rows):
        part = list(rows[off[r]:off[r + 1]])
        assert part[0] == r
        players = part[1:]
        if r < T * N * KL:
            g, f = r // (T * KL), (r % (T * KL)) // KL
            members = [p for p in range(P) if lab[f, p] == g]
            assert len(players) == len(members)
            for x in players:
                rk, i = divmod(x - t.hub_rows, slot)
                tr = tops[rk]
                src = tr.hub_partial_src()
                assert src[i] == r and tr.hp_players[rk][i // (T * KL)] in members
        else:
            assert players == []


@pytest.mark.parametrize("seed", range(6))
def test_random_strip_splits_cover_needs_and_partials(seed):
    """Random shapes and rank counts: every strip computed once, every mate
    unit a rank's strips attend to (dense mask) is local or listed in its
    needs and served by the player's home rank, and every member player of
    every local hub row has exactly one partial row."""
    from multics_b200.sharded import STRIP_ROWS, ShardTopology

    rng = np.random.default_rng(seed)
    P = int(rng.integers(2, 7))
    world = int(rng.integers(1, P + 1))
    T, L = int(rng.integers(2, 6)), int(rng.integers(20, 140))
    N, KL, KG = 2, int(rng.integers(1, 4)), int(rng.integers(0, 3))
    n_block = int(rng.choice([1, 2])) if T % 2 == 0 else 1
    lab = rng.integers(0, N, size=(T, P))
    for t0 in range(0, T, n_block):
        lab[t0:t0 + n_block] = lab[t0]
    dense = O.dense_mask(P, T, L, N, KL, KG, n_block, -1, labels=lab, direct=True)
    tops = [ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=n_block, local_attn=-1,
                          direct=True, labels=lab, world=world, rank=r) for r in range(world)]
    computed = np.zeros(P * T * L, np.int64)
    for r, t in enumerate(tops):
        rows = []
        for p, b, e in t.segments[r]:
            rows.append(p * T * L + np.arange(b * STRIP_ROWS, min(e * STRIP_ROWS, T * L)))
        rows = np.concatenate(rows)
        computed[rows] += 1
        assert set(t.local_rows()[t.computed_rows()]) == set(rows)
        cols = np.nonzero(dense[rows].any(0))[0]
        need = {(c // (T * L), (c % (T * L)) // L) for c in cols if c < P * T * L}
        need = {u for u in need if u[0] not in t.local_players}
        assert set(t.needs[r]) == need
        for o, _ in t.needs[r]:
            assert o in tops[int(t.home[o])].local_players
    assert (computed == 1).all()
    off, rows = tops[0].hub_partials()
    slot = tops[0].hub_partial_slot
    for h in range(T * N * KL):
        g, f = h // (T * KL), (h % (T * KL)) // KL
        players = []
        for x in rows[off[h] + 1:off[h + 1]]:
            rk, i = divmod(int(x) - tops[0].hub_rows, slot)
            players.append(tops[rk].hp_players[rk][i // (T * KL)])
        assert sorted(players) == [p for p in range(P) if lab[f, p] == g]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_hub_key_split_partitions_the_pairs(world):
    """The ranks' hub-key pair ranges partition every pair once, and the
    owner of each hub row is the rank whose range holds its pair."""
    from multics_b200.sharded import ShardTopology

    P, T, L, N, KL, KG = 8, 20, 40, 4, 16, 6
    lab = _regrouped_labels(P, T, 3, seed=2)
    tops = [ShardTopology(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n_block=1, local_attn=-1,
                          direct=True, labels=lab, world=world, rank=r) for r in range(world)]
    splits = [t.hub_key_split() for t in tops]
    npl, npg = -(-T * KL // 256), -(-T * KG // 256)
    covered = []
    for first, count, _ in splits:
        covered += list(range(first, first + count))
    assert covered == list(range(N * npl + npg))
    owner = splits[0][2]
    assert all(np.array_equal(owner, s[2]) for s in splits)
    h = np.arange(tops[0].hub_rows)
    for r, (first, count, _) in enumerate(splits):
        for pair in range(first, first + count):
            if pair < N * npl:
                g, j = divmod(pair, npl)
                rows = h[g * T * KL + 256 * j: min(g * T * KL + 256 * (j + 1), (g + 1) * T * KL)]
            else:
                j = pair - N * npl
                rows = T * N * KL + np.arange(256 * j, min(256 * (j + 1), T * KG))
            assert (owner[rows] == r).all()

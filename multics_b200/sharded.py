"""Player-sharded hierarchical attention: one rank per GPU over NCCL.

Each rank owns a contiguous range of whole players (uneven when the count
does not divide).  Per layer:

1. **exchange** - ranks send each other exactly the group-mate frames that
   direct player edges need (``all_to_all_single``; with static groups kept
   on one rank nothing moves);
2. **attention** - one tcgen05 launch over the rank's query rows (its
   players' rows, then every hub row, the hubs group-major) reading three
   key/value streams in place: its players' rows, the hub rows, the received
   mate frames.  Player rows run in 256-row strips, hub rows in 128-row
   tiles of one group's frames, over exactly the key units they attend to
   (per-row masks where a tile is seen in part);
3. **hub merge** - hub rows were computed over the keys each rank holds;
   their partial results merge from the per-row log-sum-exp with an
   all-reduce of the max and one all-reduce of the scaled partial sums.

Hub tokens are replicated on every rank (``T*(N*K_L+K_G)`` rows, 1.6k at the
benchmark shapes), so only mate frames and hub partials cross NVLink.
Multi-rank host logic (topology, exchange order, merge) is exercised with
``gloo`` ranks on CPU; the CUDA path requires the library.
"""

from __future__ import annotations

import ctypes
import math
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import HierPartialOut, HierShardDesc, HierShardSizes, check, ptr, stream_ptr

__all__ = ["split_players", "ShardTopology", "ShardedHierAttention", "exchange_mate_frames"]


STRIP_ROWS = 256  # query rows of one attention work item (two 128-row tiles)


def split_players(P: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous player ranges per rank, the first ``P % world`` ranks one larger."""
    if world < 1 or world > P:
        raise ValueError(f"cannot shard {P} players over {world} ranks")
    base, extra = divmod(P, world)
    out, p = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((p, p + n))
        p += n
    return out


def strip_weights(T: int, L: int, KL: int = 0) -> np.ndarray:
    """Work weight of each of a player's 256-row strips: its last frame + 2
    (its key count grows with the history it attends to).  With ``K_L`` the
    player's hub-partial strips (its group's hub rows of every frame, over
    the same history) are added to its last strip, which decides the rank
    that computes them."""
    nps = -(-T * L // STRIP_ROWS)
    w = np.array([(min((s + 1) * STRIP_ROWS, T * L) - 1) // L + 2 for s in range(nps)],
                 dtype=np.float64)
    if KL > 0:
        nph = -(-T * KL // STRIP_ROWS)
        w[-1] += sum((min((s + 1) * STRIP_ROWS, T * KL) - 1) // KL + 2 for s in range(nph))
    return w


def split_strips(P: int, T: int, L: int, world: int, KL: int = 0
                 ) -> List[List[Tuple[int, int, int]]]:
    """Balanced split of every player's 256-row strips over the ranks: the
    strips of players 0..P-1 in order, weighted by :func:`strip_weights`, cut
    into ``world`` contiguous runs of equal weight.  Returns per rank
    ``(player, first strip, end strip)`` segments; whole players per rank
    when ``world`` divides ``P``."""
    if world < 1 or world > P:
        raise ValueError(f"cannot shard {P} players over {world} ranks")
    nps = -(-T * L // STRIP_ROWS)
    weights = np.tile(strip_weights(T, L, KL), P)
    cum = np.concatenate([[0.0], np.cumsum(weights)])
    total = cum[-1]
    cuts = [0] + [int(np.argmin(np.abs(cum - total * r / world))) for r in range(1, world)] + \
        [P * nps]
    out = []
    for r in range(world):
        segs = []
        i0, i1 = cuts[r], cuts[r + 1]
        for p in range(P):
            b, e = max(i0, p * nps), min(i1, (p + 1) * nps)
            if b < e:
                segs.append((p, b - p * nps, e - p * nps))
        out.append(segs)
    return out


class ShardTopology:
    """Host-side description of one sharded layer (identical on every rank).

    ``labels``: int64 ``[T, P]`` group labels.  Work is split by 256-row
    strips (:func:`split_strips`): rank ``r`` computes ``segments[r]`` and
    holds the rows of every player it computes strips of (its *local*
    players, in increasing order).  Each player's *home* is the rank holding
    its last strip: it computes the player's hub partial rows and serves its
    frames to ranks that need them as group-mate keys.  ``needs[r]`` lists
    the units ``(o, f)`` (L rows of player ``o`` at frame ``f``) rank ``r``
    reads from another rank through direct edges, ordered by (home rank,
    player, frame): the order of its remote buffer and of the ``all_to_all``
    receive splits."""

    def __init__(self, *, P, T, L, N, KL, KG, n_block, local_attn, direct, labels, world, rank):
        self.P, self.T, self.L, self.N, self.KL, self.KG = P, T, L, N, KL, KG
        self.n_block, self.local_attn, self.direct = n_block, local_attn, bool(direct)
        self.world, self.rank = world, rank
        lab = np.asarray(labels, dtype=np.int64).reshape(T, P)
        self.labels = lab
        self.nps = -(-T * L // STRIP_ROWS)
        self.segments = split_strips(P, T, L, world, KL)
        self.local = [[p for p, _, _ in segs] for segs in self.segments]
        self.home = np.zeros(P, dtype=np.int64)
        for r, segs in enumerate(self.segments):
            for p, _, e in segs:
                if e == self.nps:
                    self.home[p] = r
        self.hp_players = [[p for p in self.local[r] if self.home[p] == r] for r in range(world)]
        self.local_players = self.local[rank]
        self.n_local = len(self.local_players)
        if self.n_local > _lib.SHARD_MAX_LOCAL:
            raise ValueError(f"a rank would hold {self.n_local} players; at most "
                             f"{_lib.SHARD_MAX_LOCAL}")
        self.hub_rows = T * (N * KL + KG)
        self.own_rows = self.n_local * T * L
        w = strip_weights(T, L, KL)
        self.work_share = sum(w[b:e].sum() for _, b, e in self.segments[rank]) / (P * w.sum())
        self.needs = [self._needs(r) for r in range(world)]
        mine = self.needs[rank]
        self.recv_units = [sum(1 for o, _ in mine if self.home[o] == i) for i in range(world)]
        self.send_units = [[u for u in self.needs[j] if self.home[u[0]] == rank]
                           for j in range(world)]
        rows = []
        for j in range(world):
            for o, f in self.send_units[j]:
                start = self.local_players.index(o) * T * L + f * L
                rows.append(np.arange(start, start + L))
        self.send_rows = (np.concatenate(rows) if rows else np.zeros(0, np.int64)).astype(np.int64)

    def remote_keys(self, transport: str) -> np.ndarray:
        """int32 ``[P*T]``: stream-packed first row of every remote unit this
        rank reads (-1 elsewhere).  ``"exchange"``: slot ``i`` of the received
        buffer (stream 2); ``"peer"``: the home rank's own rows, stream
        ``2 + j`` for the ``j``-th other rank."""
        keys = np.full(self.P * self.T, -1, dtype=np.int64)
        others = [r for r in range(self.world) if r != self.rank]
        for i, (o, f) in enumerate(self.needs[self.rank]):
            if transport == "exchange":
                keys[o * self.T + f] = (2 << 24) | (i * self.L)
            else:
                h = int(self.home[o])
                slot = self.local[h].index(o)
                keys[o * self.T + f] = ((2 + others.index(h)) << 24) | \
                    (slot * self.T * self.L + f * self.L)
        return keys.astype(np.int32)

    def _needs(self, r):
        if not self.direct:
            return []
        n, T, L = self.n_block, self.T, self.L
        local = set(self.local[r])
        units = set()
        for p, b, e in self.segments[r]:
            f_lo, f_hi = (b * STRIP_ROWS) // L, (min(e * STRIP_ROWS, T * L) - 1) // L
            for qf in range(f_lo, f_hi + 1):
                bs = (qf // n) * n
                for o in range(self.P):
                    if o == p or o in local or self.labels[qf, o] != self.labels[qf, p]:
                        continue
                    for kf in range(bs, min(bs + n, T)):
                        units.add((o, kf))
        return sorted(units, key=lambda u: (self.home[u[0]], u[0], u[1]))

    def computed_rows(self) -> np.ndarray:
        """Local rows (player slots) this rank computes: its strips' rows."""
        T, L = self.T, self.L
        rows = []
        for p, b, e in self.segments[self.rank]:
            slot = self.local_players.index(p)
            rows.append(slot * T * L + np.arange(b * STRIP_ROWS, min(e * STRIP_ROWS, T * L)))
        return np.concatenate(rows).astype(np.int64)

    def hub_rows_order(self) -> np.ndarray:
        """Sequence rows of the hub rows in the shard's order: local hubs
        group-major ``(g, f, slot)``, then the global hubs ``(f, slot)``.  A
        group's hub tokens of consecutive frames are consecutive rows, so a
        hub query tile holds one group and a player's hub keys form one run."""
        T, N, KL, KG = self.T, self.N, self.KL, self.KG
        A = self.P * T * self.L
        g_i, f_i, s_i = np.meshgrid(np.arange(N), np.arange(T), np.arange(KL), indexing="ij")
        local = A + ((f_i * N + g_i) * KL + s_i).reshape(-1)
        glob = A + T * N * KL + np.arange(T * KG)
        return np.concatenate([local, glob]).astype(np.int64)

    def local_rows(self) -> np.ndarray:
        """Sequence rows of this rank's query rows: its local players' rows
        (slot order), then every hub row in :meth:`hub_rows_order`."""
        TL = self.T * self.L
        own = [np.arange(p * TL, (p + 1) * TL) for p in self.local_players]
        return np.concatenate(own + [self.hub_rows_order()]).astype(np.int64)

    def hub_partial_src(self, r=None) -> np.ndarray:
        """Hub row (in :meth:`hub_rows_order`) of each player-partial row of
        rank ``r`` (default this rank): hub-partial player ``p`` (k-th),
        frame ``t``, slot ``s`` -> the local hub of ``p``'s group at ``t``."""
        T, KL = self.T, self.KL
        players = self.hp_players[self.rank if r is None else r]
        if not players:
            return np.zeros(0, np.int64)
        p_i, t_i, s_i = np.meshgrid(np.array(players), np.arange(T), np.arange(KL),
                                    indexing="ij")
        g = self.labels[t_i, p_i]
        return ((g * T + t_i) * KL + s_i).reshape(-1).astype(np.int64)

    def hub_key_split(self):
        """This rank's share of the hub-key pairs (one group's ``T*K_L``
        local-hub rows or the ``T*K_G`` global rows per 256-row strip, local
        groups first) as ``(first, count)``, and the rank that computes the
        hub-token partial of every hub row (group-major order), ``int32
        [hub_rows]``."""
        T, N, KL, KG, W = self.T, self.N, self.KL, self.KG, self.world
        npl = -(-T * KL // 256) if KL > 0 else 0
        npg = -(-T * KG // 256) if KG > 0 else 0
        n = N * npl + npg
        bounds = [r * n // W for r in range(W + 1)]
        rank_of = np.zeros(max(n, 1), np.int32)
        for r in range(W):
            rank_of[bounds[r]:bounds[r + 1]] = r
        h = np.arange(self.hub_rows)
        loc = T * N * KL
        pair = np.where(h < loc, (h // max(T * KL, 1)) * npl + (h % max(T * KL, 1)) // 256,
                        N * npl + (h - loc) // 256)
        owner = rank_of[np.minimum(pair, max(n, 1) - 1)].astype(np.int32)
        first = bounds[self.rank]
        return first, bounds[self.rank + 1] - first, owner

    @property
    def hub_partial_slot(self) -> int:
        """Rows of one rank's player-partial block in the shared partial-row
        buffer (the largest rank's hub-partial players x ``T*K_L``)."""
        return max(len(x) for x in self.hp_players) * self.T * self.KL

    def hub_partials(self):
        """CSR of the partial rows of every hub row, in the partial-row buffer
        every rank assembles: ``[0, hub_rows)`` the hub-token partials (each
        rank computes them), then per rank a slot of
        :attr:`hub_partial_slot` rows with its players' partials.  Returns
        ``off [hub_rows+1]`` and ``rows``."""
        T, KL = self.T, self.KL
        lists = [[r] for r in range(self.hub_rows)]
        slot = self.hub_partial_slot
        for r in range(self.world):
            for k, p in enumerate(self.hp_players[r]):
                for t in range(T):
                    g = int(self.labels[t, p])
                    base = self.hub_rows + r * slot + (k * T + t) * KL
                    for s in range(KL):
                        lists[(g * T + t) * KL + s].append(base + s)
        off = np.zeros(self.hub_rows + 1, dtype=np.int32)
        off[1:] = np.cumsum([len(x) for x in lists])
        rows = np.array([x for lst in lists for x in lst], dtype=np.int32)
        return off, rows


def _stream_arrays(streams):
    n = len(streams)
    kp = (ctypes.c_void_p * n)(*[k.data_ptr() for k, _ in streams])
    vp = (ctypes.c_void_p * n)(*[v.data_ptr() for _, v in streams])
    rows = (ctypes.c_int64 * n)(*[k.shape[0] for k, _ in streams])
    strides = (ctypes.c_int64 * n)(*[k.stride(0) for k, _ in streams])
    return n, kp, vp, rows, strides


def exchange_mate_frames(topo: ShardTopology, k, v, remote, group=None, send_rows=None):
    """``all_to_all`` of the group-mate frames each rank's direct edges need:
    rank ``j`` receives, in its ``needs`` order, the ``[K | V]`` rows of the
    units it needs into ``remote`` (``[>= units*L, 2*dim]``)."""
    t = topo
    if t.world == 1 or not t.direct:
        return remote
    import torch.distributed as dist

    rows = send_rows if send_rows is not None else torch.from_numpy(t.send_rows).to(k.device)
    dim = k.shape[1]
    send = (torch.cat([k.index_select(0, rows), v.index_select(0, rows)], dim=1)
            if rows.numel() else torch.empty((0, 2 * dim), dtype=k.dtype, device=k.device))
    n_recv = sum(t.recv_units) * t.L
    dist.all_to_all_single(remote[:n_recv], send, [n * t.L for n in t.recv_units],
                           [len(u) * t.L for u in t.send_units], group=group)
    return remote


class ShardedHierAttention:
    """One rank's sharded attention layer (inputs already projected and roped).

    ``forward(q, k, v)`` takes this rank's rows in local order (its local
    players' ``T*L`` rows each, then all ``T*(N*K_L+K_G)`` hub rows), bf16
    ``[rows, H*128]``, and returns the attention output for the same rows:
    the rows of its strips (``topo.computed_rows()``) and every hub row,
    identical on every rank after the merge; a local player's rows computed
    by another rank are left as they were in ``out``.

    ``transport`` selects how group-mate frames on other ranks are read:
    ``"exchange"`` fetches them with ``all_to_all`` before the launch;
    ``"peer"`` keeps every rank's K/V in symmetric memory and the attention
    kernel reads the other ranks' rows in place over NVLink (plain TMA loads
    of peer memory, no copy).  In peer mode K and V must be written into
    :meth:`k_buffer` / :meth:`v_buffer` (other tensors are copied there).

    ``spread_hub_keys`` (default: with the peer transport) gives each rank a
    share of the hub-token partial pairs instead of all of them; the peer
    merge then reads each hub row's hub-token partial from the rank that
    computed it (:attr:`hub_key_owner`)."""

    def __init__(self, topo: ShardTopology, num_heads: int, device, group=None,
                 transport: str = "exchange", active=None, page_table=None,
                 spread_hub_keys=None):
        if transport not in ("exchange", "peer"):
            raise ValueError(f"unknown transport {transport!r}")
        self.topo = topo
        self.H = num_heads
        self.D = 128
        self.dim = num_heads * 128
        self.device = torch.device(device)
        self.group = group
        t = topo
        dev = self.device
        self.transport = transport if (t.world > 1 and t.direct) else "exchange"
        self._labels = torch.from_numpy(t.labels).to(dev).contiguous()
        if active is None:
            act = np.zeros((t.T, t.N), dtype=np.uint8)
            for f in range(t.T):
                for p in range(t.P):
                    act[f, t.labels[f, p]] = 1
            self._active = torch.from_numpy(act).to(dev)
        else:  # the caller's active groups ([T, N]), as the reference accepts
            self._active = torch.as_tensor(active).to(device=dev, dtype=torch.uint8).contiguous()
            if tuple(self._active.shape) != (t.T, t.N):
                raise ValueError(f"active must be [T={t.T}, N={t.N}], got "
                                 f"{tuple(self._active.shape)}")
        self._keys = torch.from_numpy(t.remote_keys(self.transport)).to(dev)
        d = HierShardDesc()
        d.P, d.N, d.L, d.KL, d.KG, d.T = t.P, t.N, t.L, t.KL, t.KG, t.T
        d.n_block, d.local_attn, d.direct = t.n_block, t.local_attn, int(t.direct)
        # hub-token partials: with the peer transport the hub-key pairs are
        # spread over the ranks and the merge reads each partial from its
        # rank (hub_key_owner); otherwise every rank computes all of them, so
        # that only the per-player hub partials cross GPUs
        d.n_local, d.hub_keys = t.n_local, 1
        self.hub_key_owner = None
        spread = (self.transport == "peer") if spread_hub_keys is None else bool(spread_hub_keys)
        if spread and t.world > 1:
            first, count, owner = t.hub_key_split()
            d.hub_keys = int(count > 0)
            d.hub_key_first, d.hub_key_count = first, count
            self.hub_key_owner = torch.from_numpy(owner).to(dev)
        d.hub_partial_row0 = t.rank * t.hub_partial_slot
        for i, p in enumerate(t.local_players):
            b, e = next(((b_, e_) for p_, b_, e_ in t.segments[t.rank] if p_ == p), (0, 0))
            d.local_player[i], d.strip_begin[i], d.strip_end[i] = p, b, e
            d.hub_partials[i] = int(t.home[p] == t.rank)
        d.labels, d.active, d.remote_key = (self._labels.data_ptr(), self._active.data_ptr(),
                                            self._keys.data_ptr())
        # stream 0 (the shard's player rows) in 64-row pages: its key/value
        # tensors hold page_table[p] * 64 + r % 64 for logical row r
        self.page_rows = 0
        if page_table is not None:
            if t.world != 1:
                raise ValueError("a page table is supported on a single rank (the mate-frame "
                                 "exchange reads rows in place)")
            self._pages = torch.as_tensor(page_table).to(device=dev, dtype=torch.int32).contiguous()
            d.page_table, d.n_pages = self._pages.data_ptr(), int(self._pages.numel())
            self.page_rows = (int(self._pages.max().item()) + 1) * 64
        self.desc = d
        sz = HierShardSizes()
        lib = _lib.lib()
        check(lib.hier_shard_sizes(ctypes.byref(d), ctypes.byref(sz)))
        self.n_pairs = int(sz.n_pairs)
        self.n_player_pairs = int(sz.n_player_pairs)
        self.q_rows = int(sz.own_rows + sz.hub_rows)
        self.hp_rows = int(sz.hub_partial_rows)
        # plan: count key tiles and masks, size the tables (one host read), build
        self.counts = torch.empty(max(sz.n_counts, 1), dtype=torch.int32, device=dev)
        totals = torch.zeros(2, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        check(lib.hier_shard_count(ctypes.byref(d), ptr(self.counts), ptr(totals),
                                   ptr(self.status), stream_ptr(dev)))
        n_tiles, n_masks = (int(x) for x in totals.cpu())
        self.n_tiles, self.n_masks = n_tiles, n_masks
        self.q_pairs = torch.empty((max(self.n_pairs, 1), 8), dtype=torch.int32, device=dev)
        self.kv_tiles = torch.empty((max(n_tiles, 1), 4), dtype=torch.int32, device=dev)
        self.tile_masks = torch.empty((max(n_masks, 1), 128, 4), dtype=torch.int32, device=dev)
        self.order = torch.empty(max(self.n_pairs, 1), dtype=torch.int32, device=dev)
        check(lib.hier_shard_build(ctypes.byref(d), ptr(self.counts), ptr(self.q_pairs),
                                   ptr(self.kv_tiles), max(n_tiles, 1), ptr(self.tile_masks),
                                   max(n_masks, 1), ptr(self.order), ptr(self.status),
                                   stream_ptr(dev)))
        self.send_rows = torch.from_numpy(t.send_rows).to(dev)
        self.n_recv = sum(t.recv_units) * t.L if self.transport == "exchange" else 0
        self.remote = torch.zeros((max(self.n_recv, 1), 2 * self.dim), dtype=torch.bfloat16,
                                  device=dev)
        # hub rows as partial rows: the hub-token part, then one slot per rank
        # for its home players' partials (read in place from the other ranks
        # with the peer transport, all-gathered in place otherwise)
        slot = t.hub_partial_slot
        n_part = t.hub_rows + t.world * slot
        self.part_o = torch.zeros((max(n_part, 1), self.dim), dtype=torch.bfloat16, device=dev)
        self.part_lse = torch.full((max(n_part, 1), self.H), float("-inf"), dtype=torch.float32,
                                   device=dev)
        self.q_hp = torch.empty((max(self.hp_rows, 1), self.dim), dtype=torch.bfloat16,
                                device=dev)
        self.hp_src = torch.from_numpy(t.hub_partial_src()).to(dev)
        off, rows = t.hub_partials()
        self.csr_off = torch.from_numpy(off).to(dev)
        self.csr_rows = torch.from_numpy(rows if rows.size else np.zeros(1, np.int32)).to(dev)
        from .attention import _dev_err
        self.err = _dev_err(dev)
        self._sym = None
        self._peers = []
        # a plan whose tables overflowed is refused here, before any launch
        self.check_status()
        if self.transport == "peer":
            self._setup_peer()

    def _setup_peer(self):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        t = self.topo
        group = self.group if self.group is not None else dist.group.WORLD
        if hasattr(symm, "enable_symm_mem_for_group"):
            try:
                symm.enable_symm_mem_for_group(group.group_name)
            except Exception:  # already enabled / not needed in this torch version
                pass
        rows = max(len(x) for x in t.local) * t.T * t.L + t.hub_rows
        self._sym_rows = rows
        self._sym = symm.empty((2, rows, self.dim), dtype=torch.bfloat16, device=self.device)
        self._sym.zero_()
        self._handle = symm.rendezvous(self._sym, group)
        for r in range(t.world):
            if r == t.rank:
                continue
            buf = self._handle.get_buffer(r, (2, rows, self.dim), torch.bfloat16)
            n = len(t.local[r]) * t.T * t.L
            self._peers.append((buf[0, :n], buf[1, :n]))
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        # hub partial rows in symmetric memory too: the merge reads the other
        # ranks' player partials in place
        shape_o, shape_l = tuple(self.part_o.shape), tuple(self.part_lse.shape)
        self.part_o = symm.empty(shape_o, dtype=torch.bfloat16, device=self.device)
        self.part_lse = symm.empty(shape_l, dtype=torch.float32, device=self.device)
        self.part_o.zero_()
        self.part_lse.fill_(float("-inf"))
        h_o = symm.rendezvous(self.part_o, group)
        h_l = symm.rendezvous(self.part_lse, group)
        self._part_handles = (h_o, h_l)
        o_bases, l_bases = [], []
        self._part_peers = []
        for r in range(t.world):
            if r == t.rank:
                po, pl = self.part_o, self.part_lse
            else:
                po = h_o.get_buffer(r, shape_o, torch.bfloat16)
                pl = h_l.get_buffer(r, shape_l, torch.float32)
                self._part_peers.append((po, pl))
            o_bases.append(po.data_ptr())
            l_bases.append(pl.data_ptr())
        self._part_o_bases = torch.tensor(o_bases, dtype=torch.int64, device=self.device)
        self._part_lse_bases = torch.tensor(l_bases, dtype=torch.int64, device=self.device)

    def k_buffer(self):
        """Where K of this rank's rows should be written (peer transport)."""
        return self._sym[0, :self.q_rows] if self._sym is not None else None

    def v_buffer(self):
        return self._sym[1, :self.q_rows] if self._sym is not None else None

    def check_status(self):
        st = int(self.status.item())
        if st:
            raise RuntimeError(f"sharded plan status {st:#x} (8: missing remote unit, "
                               "2: tile capacity, 16: mask capacity)")

    def exchange(self, k, v):
        """Make the other ranks' mate frames readable: fetch them
        (``exchange``) or order the peer reads after every rank's writes
        (``peer``: a one-element all-reduce on the stream)."""
        if self.transport == "peer":
            import torch.distributed as dist

            if k.data_ptr() != self.k_buffer().data_ptr():
                self.k_buffer().copy_(k)
            if v.data_ptr() != self.v_buffer().data_ptr():
                self.v_buffer().copy_(v)
            dist.all_reduce(self._flag, group=self.group)
            return
        exchange_mate_frames(self.topo, k, v, self.remote, self.group, self.send_rows)

    def fill_remote_from(self, k_all, v_all):
        """Single-process stand-in for :meth:`exchange`: copy the needed mate
        frames from full-sequence K/V (tests emulating several ranks)."""
        t = self.topo
        for i, (o, f) in enumerate(t.needs[t.rank]):
            src = (o * t.T + f) * t.L
            self.remote[i * t.L:(i + 1) * t.L, :self.dim] = k_all[src:src + t.L]
            self.remote[i * t.L:(i + 1) * t.L, self.dim:] = v_all[src:src + t.L]

    def attend(self, q, k, v, out, *, v_hub=None, out_rows=None, lse=None):
        """One attention launch over this rank's query rows: player rows into
        ``out`` (row ``out_rows[r]`` when given), hub rows as partial rows
        (merged by :meth:`merge`).  ``v_hub`` replaces ``v``'s hub rows (a
        group-major copy when ``v`` keeps the sequence order).  ``lse``
        (float32 ``[rows, H]``, optional) receives the player rows'
        log2-sum-exp at the same rows as ``out``; the hub rows' partials keep
        theirs in :attr:`part_lse`."""
        t = self.topo
        own, hub = t.own_rows, t.hub_rows
        if self.transport == "peer":
            k, v = self.k_buffer(), self.v_buffer()
        if self.n_pairs == 0:
            return
        if self.hp_rows:
            torch.index_select(q[own:own + hub], 0, self.hp_src, out=self.q_hp)
        # key/value streams: player rows (in place, or a pool of pages), hub rows
        n0 = self.page_rows or own
        streams = [(k[:n0], v[:n0]),
                   (k[n0:n0 + hub], v[n0:n0 + hub] if v_hub is None else v_hub)]
        if self.transport == "peer":
            streams += self._peers
        else:
            streams.append((self.remote[:, :self.dim], self.remote[:, self.dim:]))
        n, kp, vp, rows, strides = _stream_arrays(streams)
        part = HierPartialOut()
        part.q2, part.q2_rows, part.q2_stride = self.q_hp.data_ptr(), self.q_hp.shape[0], \
            self.q_hp.stride(0)
        part.q2_row0 = own + hub + t.rank * t.hub_partial_slot
        part.o, part.o_stride = self.part_o.data_ptr(), self.part_o.stride(0)
        part.lse, part.row0 = self.part_lse.data_ptr(), own
        check(_lib.lib().hier_attn_fwd_streams(
            ptr(q), q.shape[0], q.stride(0), n, kp, vp, rows, strides, ptr(out), out.stride(0),
            ptr(out_rows), self.H, self.D, ptr(self.q_pairs), self.n_pairs, ptr(self.kv_tiles),
            ptr(self.tile_masks), 128, ptr(self.order), 1.0 / math.sqrt(self.D), ptr(lse),
            ctypes.byref(part), ptr(self.err), stream_ptr(q.device)))

    # ---- hub merge: partial rows -> hub rows ---------------------------------
    def gather_partials(self):
        """All-gather every rank's player-partial slot (rows and log-sum-exp)
        into this rank's partial-row buffer, in place."""
        t = self.topo
        if t.world == 1 or t.hub_partial_slot == 0:
            return
        import torch.distributed as dist

        h0, slot = t.hub_rows, t.hub_partial_slot
        o_all = self.part_o[h0:h0 + t.world * slot]
        l_all = self.part_lse[h0:h0 + t.world * slot]
        r0 = t.rank * slot
        dist.all_gather_into_tensor(o_all, o_all[r0:r0 + slot], group=self.group)
        dist.all_gather_into_tensor(l_all, l_all[r0:r0 + slot], group=self.group)

    def merge_partials(self, out_hub, out_rows=None):
        """Merged hub rows from the assembled partial-row buffer into
        ``out_hub`` (``[hub_rows, H*D]``, or rows ``out_rows[r]`` of it)."""
        t = self.topo
        check(_lib.lib().hier_lse_gather_merge(
            ptr(self.part_o), self.part_o.stride(0), ptr(self.part_lse), self.H, self.D,
            ptr(self.csr_off), ptr(self.csr_rows), t.hub_rows, ptr(out_hub), out_hub.stride(0),
            ptr(out_rows), stream_ptr(self.device)))
        return out_hub

    def merge(self, out_hub, out_rows=None):
        """Hub rows: one gather kernel merges every hub row's partials by
        log-sum-exp.  With the peer transport it reads the other ranks'
        player partials in place after a one-element all-reduce (every rank's
        partials written); otherwise they are all-gathered first."""
        t = self.topo
        if t.hub_rows == 0:
            return out_hub
        if self.hub_key_owner is not None and self.transport != "peer":
            raise RuntimeError("hub-token partials spread over the ranks need the peer merge")
        if t.world > 1 and self.transport == "peer":
            import torch.distributed as dist

            dist.all_reduce(self._flag, group=self.group)
            check(_lib.lib().hier_lse_gather_merge_peers(
                ptr(self._part_o_bases), ptr(self._part_lse_bases), t.world, t.rank, t.hub_rows,
                max(t.hub_partial_slot, 1), self.part_o.stride(0), self.H, self.D,
                ptr(self.csr_off), ptr(self.csr_rows), t.hub_rows, ptr(out_hub),
                out_hub.stride(0), ptr(out_rows), ptr(self.hub_key_owner),
                stream_ptr(self.device)))
            return out_hub
        self.gather_partials()
        return self.merge_partials(out_hub, out_rows)

    def forward(self, q, k, v, out=None, events=None):
        """The layer's attention over this rank's rows: exchange, one
        attention launch, hub merge (:meth:`merge`).
        ``events`` (optional, two CUDA events) are recorded after the
        exchange and after the attention launch.  (Running the hub pairs as a
        first launch with the all-gather overlapping the player strips was
        slower at 8 GPUs: 1.09 against 1.06 ms per config-4 layer.)"""
        t = self.topo
        kv_rows = (self.page_rows or t.own_rows) + t.hub_rows
        if q.shape != (self.q_rows, self.dim) or k.shape != (kv_rows, self.dim) or \
                v.shape != k.shape:
            raise ValueError(f"expected query rows [{self.q_rows}, {self.dim}] and key/value "
                             f"rows [{kv_rows}, {self.dim}], got "
                             f"{tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
        if out is None:
            out = torch.empty_like(q)
        main = torch.cuda.current_stream(self.device)
        self.exchange(k, v)
        if events is not None:
            events[0].record(main)
        self.attend(q, k, v, out)
        if events is not None:
            events[1].record(main)
        self.merge(out[t.own_rows:])
        return out

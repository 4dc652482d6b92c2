"""Cached-step hierarchical attention on B200: the ``WAN_HIER_INFER_KERNEL``
backends of the reference's ``causal_forward_hier_hub``.

Reference-mirror entry points (same keyword arguments, outputs and error
types/messages):

* :func:`build_metadata` - ``_build_metadata``
  (``multics/models/kernels/hier_segmented_attention.py:156-395``), built on
  the device and bit-exact: ``(prog_qbase, prog_nq, prog_seg, kv_index,
  kv_count, logical_pairs)``;
* :func:`get_varlen_plan` - ``_get_varlen_plan``
  (``multics/models/kernels/hier_packed_attention.py:32-102``);
* :func:`hierarchical_cached_attention` - the cached-backend plugin signature
  shared by ``hierarchical_segmented_attention``,
  ``hierarchical_tiled_cached_attention``,
  ``hierarchical_packed_varlen_attention`` and
  ``hierarchical_paged_kv_attention`` (``hier_paged_attention.py:79-106``):
  roped queries of one cached step against the per-player, per-group and
  global rolling caches, read in place by the tcgen05 attention kernel (no
  pool concatenation, no host synchronisation).

Every path requires the CUDA library; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import math
import os
from collections import OrderedDict
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import (HierCachedGrouping, HierCachedPackSizes, HierCachedSizes, HierPartialOut,
                   check, ptr, stream_ptr)

__all__ = ["build_metadata", "get_varlen_plan", "hierarchical_cached_attention",
           "clear_metadata_cache", "CachedPlan", "build_cached_plan"]

_META_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()
_PLAN_CACHE: "OrderedDict[tuple, dict]" = OrderedDict()
_DEV_ERR = {}

# Synchronous status checks after the plan builders (membership frame range,
# plan capacity); off by default so that a cached step never waits on the GPU.
SYNC_CHECKS = os.environ.get("MULTICS_B200_SYNC_CHECKS", "0") == "1"


def _dev_err(device):
    key = torch.device(device).index
    t = _DEV_ERR.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _DEV_ERR[key] = t
    return t


def clear_metadata_cache():
    _META_CACHE.clear()
    _PLAN_CACHE.clear()


def _cache_limit(var, default):
    return max(int(os.environ.get(var, str(default))), 0)


def _lru_put(cache, key, value, limit):
    if limit == 0:
        return
    cache[key] = value
    cache.move_to_end(key)
    while len(cache) > limit:
        cache.popitem(last=False)


class _Grouping:
    """``hier_cached_grouping`` plus the tensors it points at (kept alive)."""

    def __init__(self, *, P, N, L, KL, KG, n_frames, n_block, local_attn, direct, no_local,
                 agent_frames, local_frames, local_active, global_frames, labels, q_active,
                 membership, global_only):
        if P > _lib.MAX_KV_STREAMS or N > _lib.MAX_KV_STREAMS:
            raise ValueError(f"at most {_lib.MAX_KV_STREAMS} players and groups; got P={P}, N={N}")
        self.keep = [agent_frames, local_frames, local_active, global_frames, labels, q_active,
                     membership, global_only]
        g = HierCachedGrouping()
        g.P, g.N, g.L, g.KL, g.KG = P, N, L, KL, KG
        g.n_frames, g.n_block, g.local_attn = n_frames, n_block, local_attn
        g.direct, g.no_local = int(bool(direct)), int(bool(no_local))
        g.membership_mode = int(membership is not None)
        g.fa = agent_frames[0].numel() // L if agent_frames else 0
        g.fl = (local_frames[0].numel() // KL) if (local_frames and KL > 0) else 0
        g.fg = (global_frames.numel() // KG) if (global_frames is not None and KG > 0) else 0
        g.T_mem = membership.shape[0] if membership is not None else 0
        for i, t in enumerate(agent_frames):
            g.agent_frames[i] = t.data_ptr()
        for i, t in enumerate(local_frames):
            g.local_frames[i] = t.data_ptr()
        for i, t in enumerate(local_active):
            g.local_active[i] = t.data_ptr()
        g.global_frames = global_frames.data_ptr() if global_frames is not None else None
        g.labels = labels.data_ptr() if labels is not None else None
        g.q_active = q_active.data_ptr()
        g.membership = membership.data_ptr() if membership is not None else None
        g.global_only = global_only.data_ptr() if global_only is not None else None
        self.c = g

    def ref(self):
        import ctypes
        return ctypes.byref(self.c)

    def sizes(self, block_m):
        out = HierCachedSizes()
        import ctypes
        check(_lib.lib().hier_cached_sizes(self.ref(), int(block_m), ctypes.byref(out)))
        return out


def _flat(t, dtype):
    """Contiguous 1-D device copy-free view (converted if needed)."""
    t = t.reshape(-1)
    if t.dtype != dtype:
        t = t.to(dtype)
    return t.contiguous()


# ---------------------------------------------------------------------------
# _build_metadata
# ---------------------------------------------------------------------------


def _validate_metadata_args(agent_frame_lists, local_frame_lists, local_active_frames,
                            global_frame_list, KL, KG, n_frames, membership, global_only,
                            no_local):
    """The checks of ``_build_metadata`` (hier_segmented_attention.py:211-267)."""
    if not agent_frame_lists or any(len(x) != len(agent_frame_lists[0])
                                    for x in agent_frame_lists):
        raise ValueError("segmented hierarchical attention requires equal agent cache lengths")
    if no_local:
        if KL != 0 or local_frame_lists or local_active_frames:
            raise ValueError("hier_no_local_hub metadata requires K_L=0 and empty local caches")
    elif not local_frame_lists or any(len(x) != len(local_frame_lists[0])
                                      for x in local_frame_lists):
        raise ValueError("segmented hierarchical attention requires equal local cache lengths")
    if membership is not None and global_only is None:
        raise ValueError("membership metadata requires global_only")
    q = tuple(global_frame_list[-n_frames:]) if KG > 0 else ()
    if len(q) != n_frames:
        q = tuple(agent_frame_lists[0][-n_frames:])
    if len(q) != n_frames:
        raise ValueError("segmented hierarchical attention cannot identify the current query frames")


def build_metadata(*, device, P, N, L, KL, KG, n_frames, n_block, local_attn, agent_frame_lists,
                   local_frame_lists, global_frame_list, local_active_frames, labels, q_active,
                   direct_player, block_m, membership=None, global_only=None,
                   hier_no_local_hub=False):
    """``_build_metadata`` with host frame tuples, built by the device kernels.

    Returns ``(prog_qbase, prog_nq, prog_seg, kv_index, kv_count,
    logical_pairs)``: int32 device tensors (kv_index ``[n_seg,
    ceil64(max count)]``, zero padded) and the logical pair count.  Results
    are LRU-cached by the same key as the reference
    (``WAN_HIER_SEGMENTED_META_CACHE_SIZE``, default 64)."""
    no_local = bool(hier_no_local_hub)
    _validate_metadata_args(agent_frame_lists, local_frame_lists, local_active_frames,
                            global_frame_list, KL, KG, n_frames, membership, global_only, no_local)
    mem_t = None if membership is None else tuple(
        tuple(tuple(bool(v) for v in pr) for pr in gr) for gr in membership)
    go_t = None if global_only is None else tuple(tuple(bool(v) for v in r) for r in global_only)
    key = (str(device), P, N, L, KL, KG, n_frames, n_block, local_attn,
           tuple(tuple(x) for x in agent_frame_lists),
           tuple(tuple(x) for x in local_frame_lists), tuple(global_frame_list),
           tuple(tuple(x) for x in local_active_frames),
           None if labels is None else tuple(tuple(r) for r in labels),
           tuple(tuple(r) for r in q_active), bool(direct_player), no_local, block_m, mem_t, go_t)
    hit = _META_CACHE.get(key)
    if hit is not None:
        _META_CACHE.move_to_end(key)
        return hit
    dev = torch.device(device)
    if dev.type != "cuda":
        raise NotImplementedError("the B200 metadata builder runs on CUDA devices only")

    def frames_tensor(frames, width):
        t = torch.tensor(list(frames), dtype=torch.int64)
        return t.repeat_interleave(max(width, 1)).to(dev)

    agent = [frames_tensor(f, L) for f in agent_frame_lists]
    local = [] if no_local else [frames_tensor(f, KL) for f in local_frame_lists]
    lact = [] if no_local else [
        torch.tensor([bool(a) for a in acts], dtype=torch.uint8).repeat_interleave(KL).to(dev)
        for acts in local_active_frames]
    glob = frames_tensor(global_frame_list, KG) if KG > 0 else torch.zeros(0, dtype=torch.int64,
                                                                          device=dev)
    lab = None if labels is None else torch.tensor([list(r) for r in labels], dtype=torch.int64,
                                                   device=dev).reshape(n_frames, P)
    qact = torch.tensor([[bool(v) for v in r] for r in q_active], dtype=torch.uint8,
                        device=dev).reshape(n_frames, max(N, 0))
    mem = None if mem_t is None else torch.tensor(mem_t, dtype=torch.uint8, device=dev)
    go = None if go_t is None else torch.tensor(go_t, dtype=torch.uint8, device=dev)
    if mem is not None:
        mem = mem.reshape(-1, N, P).contiguous()
        go = go.reshape(-1, P).contiguous()
    g = _Grouping(P=P, N=N, L=L, KL=KL, KG=KG, n_frames=n_frames, n_block=n_block,
                  local_attn=local_attn, direct=direct_player, no_local=no_local,
                  agent_frames=agent, local_frames=local, local_active=lact, global_frames=glob,
                  labels=lab, q_active=qact, membership=mem, global_only=go)
    if mem is not None:
        # the reference indexes membership[qf] / global_only[kf] by absolute frame
        frames = [f for fl in agent_frame_lists for f in fl] + list(global_frame_list)
        if frames and (min(frames) < 0 or max(frames) >= mem.shape[0]):
            raise IndexError("list index out of range")
    result = _build(g, block_m, dev, exact_width=True)
    _lru_put(_META_CACHE, key, result, _cache_limit("WAN_HIER_SEGMENTED_META_CACHE_SIZE", 64))
    return result


def _build(g: _Grouping, block_m, dev, exact_width):
    sz = g.sizes(block_m)
    L = _lib.lib()
    s = stream_ptr(dev)
    kv_count = torch.zeros(sz.n_seg, dtype=torch.int32, device=dev)
    n_boxes = torch.zeros(sz.n_seg, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(L.hier_cached_count(g.ref(), ptr(kv_count), ptr(n_boxes), ptr(status), s))
    counts = kv_count.cpu()
    if int(status.item()) & 1:
        raise IndexError("list index out of range")
    max_k = max(int(counts.max()) if counts.numel() else 1, 1)
    width = math.ceil(max_k / 64) * 64
    prog_qbase = torch.empty(sz.n_prog, dtype=torch.int32, device=dev)
    prog_nq = torch.empty_like(prog_qbase)
    prog_seg = torch.empty_like(prog_qbase)
    kv_index = torch.empty((sz.n_seg, width), dtype=torch.int32, device=dev)
    check(L.hier_cached_build(g.ref(), int(block_m), None, ptr(prog_qbase), ptr(prog_nq),
                              ptr(prog_seg), ptr(kv_index), width, None, None, None, 0, None,
                              ptr(status), s))
    P, n = g.c.P, g.c.n_frames
    ql = [g.c.L] * (P * n) + ([] if g.c.no_local else [g.c.KL] * (n * g.c.N)) + [g.c.KG] * n
    pairs = int(sum(q * int(c) for q, c in zip(ql, counts.tolist())))
    return prog_qbase, prog_nq, prog_seg, kv_index, kv_count, pairs


# ---------------------------------------------------------------------------
# _get_varlen_plan
# ---------------------------------------------------------------------------


def get_varlen_plan(*, kv_index, kv_count, qbase, qlen, seg_ids, query_tokens):
    """``_get_varlen_plan``: the packed varlen plan, built by device kernels.

    Same dict keys (``q_index``, ``k_index`` int64, ``cu_q``, ``cu_k``
    int32, ``max_q``, ``max_k``, ``min_k_index``, ``max_k_index``,
    ``metadata_sources``) plus ``page_indices`` (int32 ``k_index``, the page
    table of page size 1 of ``hier_paged_attention.py:232-249``), cached by
    the input data pointers like the reference."""
    key = (str(kv_index.device), kv_index.data_ptr(), kv_count.data_ptr(), qbase.data_ptr(),
           qlen.data_ptr(), seg_ids.data_ptr(), int(query_tokens))
    hit = _PLAN_CACHE.get(key)
    if hit is not None:
        _PLAN_CACHE.move_to_end(key)
        return hit
    qb = [int(x) for x in qbase.cpu().tolist()]
    qn = [int(x) for x in qlen.cpu().tolist()]
    si = [int(x) for x in seg_ids.cpu().tolist()]
    nk = [int(x) for x in kv_count.cpu().tolist()]
    if si != list(range(len(si))):
        raise AssertionError("packed metadata must contain exactly one program per segment")
    pos = 0
    for b, ln in zip(qb, qn):
        if b != pos:
            raise AssertionError("packed query segments must partition the query sequence exactly")
        pos += ln
    if pos != int(query_tokens):
        raise AssertionError("packed query segments must partition the query sequence exactly")
    dev = kv_index.device
    act = [s for s in si if qn[s] > 0 and nk[s] > 0]
    sum_q = sum(qn[s] for s in act)
    sum_k = sum(nk[s] for s in act)
    n_seg = len(si)
    lib = _lib.lib()
    import ctypes
    ws_bytes = ctypes.c_size_t()
    check(lib.hier_varlen_workspace_size(n_seg, ctypes.byref(ws_bytes)))
    ws = torch.empty(max(int(ws_bytes.value), 16), dtype=torch.uint8, device=dev)
    q_index = torch.empty(sum_q, dtype=torch.int64, device=dev)
    k_index = torch.empty(sum_k, dtype=torch.int64, device=dev)
    page_indices = torch.empty(sum_k, dtype=torch.int32, device=dev)
    cu_q = torch.empty(len(act) + 1, dtype=torch.int32, device=dev)
    cu_k = torch.empty(len(act) + 1, dtype=torch.int32, device=dev)
    scalars = torch.zeros(5, dtype=torch.int64, device=dev)
    kvi = kv_index.to(torch.int32).contiguous()
    check(lib.hier_varlen_plan_build(ptr(qbase.to(torch.int32).contiguous()),
                                     ptr(qlen.to(torch.int32).contiguous()), ptr(kvi),
                                     kvi.shape[1], ptr(kv_count.to(torch.int32).contiguous()),
                                     n_seg, ptr(ws), ptr(q_index), ptr(k_index), ptr(cu_q),
                                     ptr(cu_k), ptr(page_indices), ptr(scalars), stream_ptr(dev)))
    sc = scalars.cpu().tolist()
    result = {
        "q_index": q_index, "k_index": k_index, "cu_q": cu_q, "cu_k": cu_k,
        "max_q": int(sc[0]), "max_k": int(sc[1]), "min_k_index": int(sc[2]),
        "max_k_index": int(sc[3]), "page_indices": page_indices,
        "metadata_sources": (kv_index, kv_count, qbase, qlen, seg_ids),
    }
    _lru_put(_PLAN_CACHE, key, result, _cache_limit("WAN_HIER_PACKED_PLAN_CACHE_SIZE", 64))
    return result


# ---------------------------------------------------------------------------
# attention plan + plugin
# ---------------------------------------------------------------------------


# Packed hub rows in the cached attention plan (hier_cached_pack_build): on
# unless this variable is "0".
CACHED_PACK_ENV = "MULTICS_B200_CACHED_PACK"

# Split-KV of the cached step's attention: every query pair runs as this
# many CTAs over consecutive parts of its key list, merged by log-sum-exp
# ("1": no split).
CACHED_SPLIT_ENV = "MULTICS_B200_CACHED_SPLIT"

# (P, N, L, KL, KG, n, device) -> (packed row sources, output row map)
_PACK_ROWS = {}
# (q_rows, packed, chunks, device) -> (merge CSR offsets, partial rows)
_SPLIT_CSR = {}


class CachedPlan:
    """Device attention plan of one cached step (see hier_cached_build and
    hier_cached_pack_build).  With packed hub rows, ``q2_src`` lists the
    query rows read as the second query block and ``out_rows`` maps every
    query row (then every packed row) to its output row."""

    def __init__(self, q_pairs, kv_tiles, tile_masks, order, n_pairs, n_streams, status, grouping,
                 q2_src=None, out_rows=None):
        self.q_pairs = q_pairs
        self.kv_tiles = kv_tiles
        self.tile_masks = tile_masks
        self.order = order
        self.n_pairs = n_pairs
        self.n_streams = n_streams
        self.status = status
        self.grouping = grouping
        self.q2_src = q2_src
        self.out_rows = out_rows


def _pack_rows(g: _Grouping, q_rows: int, device):
    """Sequence rows of the packed hub rows (group-major local hubs, then the
    global hubs, frame-major inside a pack) and the output row map."""
    c = g.c
    key = (c.P, c.N, c.L, c.KL, c.KG, c.n_frames, str(device))
    hit = _PACK_ROWS.get(key)
    if hit is None:
        P, N, L, KL, KG, n = c.P, c.N, c.L, c.KL, c.KG, c.n_frames
        aq, lq = P * n * L, n * N * KL
        src = [aq + (f * N + gi) * KL + sl for gi in range(N) for f in range(n) for sl in range(KL)]
        src += [aq + lq + f * KG + sl for f in range(n) for sl in range(KG)]
        src_t = torch.tensor(src, dtype=torch.int64, device=device)
        rows = torch.cat([torch.arange(q_rows, dtype=torch.int32, device=device),
                          src_t.to(torch.int32)])
        hit = (src_t, rows)
        _PACK_ROWS[key] = hit
    return hit


def _split_csr(q_rows: int, q2_src, chunks: int, device):
    """Merge CSR of a split plan: output row t gathers its ``chunks`` partial
    rows, at query index t (or, for a packed hub row, the index of its
    packed copy) in every slot of ``q_rows + packed rows`` rows."""
    n2 = 0 if q2_src is None else int(q2_src.numel())
    key = (q_rows, n2, chunks, str(device), None if q2_src is None else q2_src.data_ptr())
    hit = _SPLIT_CSR.get(key)
    if hit is None:
        qi = torch.arange(q_rows, dtype=torch.int64, device=device)
        if n2:
            qi[q2_src] = q_rows + torch.arange(n2, dtype=torch.int64, device=device)
        slot = q_rows + n2
        rows = (qi[:, None] + slot * torch.arange(chunks, device=device)[None]).reshape(-1)
        off = torch.arange(q_rows + 1, dtype=torch.int32, device=device) * chunks
        hit = (off, rows.to(torch.int32).contiguous(), slot)
        _SPLIT_CSR[key] = hit
    return hit


def build_cached_plan(g: _Grouping, device, pack=None) -> CachedPlan:
    """The step's attention plan: one query pair per player segment over its
    key runs and, when the shape allows it (``pack`` None: unless
    ``MULTICS_B200_CACHED_PACK=0``), the hub rows packed per group across the
    query frames; otherwise one pair per hub segment."""
    sz = g.sizes(1)
    lib = _lib.lib()
    s = stream_ptr(device)
    ps = HierCachedPackSizes()
    check(lib.hier_cached_pack_sizes(g.ref(), ctypes.byref(ps)))
    if pack is None:
        pack = os.environ.get(CACHED_PACK_ENV, "1") != "0"
    pack = bool(pack) and ps.n_packs > 0
    status = torch.zeros(1, dtype=torch.int32, device=device)
    q_pairs = torch.empty((max(sz.n_pairs, 1), 8), dtype=torch.int32, device=device)
    cap = max(sz.tile_capacity, 1)
    mask_base = (cap + 127) // 128
    n_tiles = cap + (ps.tile_capacity if pack else 0)
    n_masks = (mask_base + ps.tile_capacity) * 128 if pack else cap
    kv_tiles = torch.empty((n_tiles, 4), dtype=torch.int32, device=device)
    tile_masks = torch.empty((n_masks, 4), dtype=torch.int32, device=device)
    order = torch.empty(max(sz.n_pairs, 1), dtype=torch.int32, device=device)
    # no count launch: each segment's tiles sit at a fixed stride of the capacity
    check(lib.hier_cached_build(g.ref(), 1, None, None, None, None, None, 0, ptr(q_pairs),
                                ptr(kv_tiles), ptr(tile_masks), cap,
                                None if pack else ptr(order), ptr(status), s))
    if not pack:
        return CachedPlan(q_pairs, kv_tiles, tile_masks, order, sz.n_pairs, sz.n_streams,
                          status, g)
    check(lib.hier_cached_pack_build(g.ref(), None, cap, n_tiles, mask_base, int(sz.q_rows),
                                     ptr(q_pairs), ptr(kv_tiles), ptr(tile_masks), ptr(order),
                                     ptr(status), s))
    q2_src, out_rows = _pack_rows(g, int(sz.q_rows), device)
    return CachedPlan(q_pairs, kv_tiles, tile_masks, order, ps.agent_pairs + ps.n_packs,
                      sz.n_streams, status, g, q2_src, out_rows)


def _kv_rows(t, name):
    """[B=1, rows, H*D] bf16 -> [rows, H*D] view with a TMA-compatible layout."""
    if t.dim() == 3:
        if t.shape[0] != 1:
            raise NotImplementedError(f"cached hierarchical attention supports B=1; got {name} "
                                      f"batch {t.shape[0]}")
        t = t[0]
    if t.dtype != torch.bfloat16:
        raise NotImplementedError(f"{name} must be bf16; got {t.dtype}")
    if t.numel() and (t.stride(-1) != 1 or (t.stride(0) * 2) % 16 or t.data_ptr() % 16):
        t = t.contiguous()
    return t


def hierarchical_cached_attention(*, roped_q, agent_frames, agent_keys, agent_vals, local_frames,
                                  local_keys, local_vals, local_active_tokens, global_frames,
                                  global_keys, global_vals, labels, active, P, N, L, KL, KG,
                                  n_frames, n_block, local_attn, direct_player, membership=None,
                                  global_only=None, hier_no_local_hub=False, sync_checks=None):
    """Cached-backend plugin (``hier_paged_attention.py:79-106`` signature).

    ``roped_q [1,S,H,128]`` bf16 against the rolling caches (lists of
    ``[1, rows, H*128]`` bf16), the same logical edges as ``_build_metadata``.
    Returns ``[1, S, H*128]`` bf16; rows without keys are 0."""
    b, s, heads, head_dim = roped_q.shape
    if b != 1 or head_dim != 128 or roped_q.dtype != torch.bfloat16:
        raise NotImplementedError(
            "B200 cached hierarchical inference requires B=1, BF16, head_dim=128; "
            f"got B={b}, dtype={roped_q.dtype}, head_dim={head_dim}")
    if not roped_q.is_cuda:
        raise NotImplementedError("B200 cached hierarchical inference requires CUDA")
    if roped_q.requires_grad:
        raise RuntimeError("B200 cached hierarchical attention is inference-only")
    if membership is not None and global_only is None:
        raise ValueError("membership requires global_only")
    no_local = bool(hier_no_local_hub)
    dev = roped_q.device
    if not agent_frames or any(f.numel() != agent_frames[0].numel() for f in agent_frames):
        raise ValueError("segmented hierarchical attention requires equal agent cache lengths")
    if no_local:
        if KL != 0 or local_frames or local_active_tokens:
            raise ValueError("hier_no_local_hub metadata requires K_L=0 and empty local caches")
    elif not local_frames or any(f.numel() != local_frames[0].numel() for f in local_frames):
        raise ValueError("segmented hierarchical attention requires equal local cache lengths")
    agent = [_flat(f, torch.int64) for f in agent_frames]
    local = [] if no_local else [_flat(f, torch.int64) for f in local_frames]
    lact = [] if no_local else [_flat(a, torch.bool).view(torch.uint8) for a in local_active_tokens]
    glob = _flat(global_frames, torch.int64) if KG > 0 else None
    lab = None if labels is None else labels.to(device=dev, dtype=torch.int64).reshape(
        n_frames, P).contiguous()
    qact = active.to(device=dev, dtype=torch.bool).reshape(n_frames, N).contiguous().view(
        torch.uint8)
    mem = go = None
    if membership is not None:
        mem = membership.to(device=dev, dtype=torch.bool).contiguous().view(torch.uint8)
        go = global_only.to(device=dev, dtype=torch.bool).contiguous().view(torch.uint8)
    g = _Grouping(P=P, N=N, L=L, KL=KL, KG=KG, n_frames=n_frames, n_block=n_block,
                  local_attn=local_attn, direct=direct_player, no_local=no_local,
                  agent_frames=agent, local_frames=local, local_active=lact, global_frames=glob,
                  labels=lab, q_active=qact, membership=mem, global_only=go)
    plan = build_cached_plan(g, dev)
    keys = list(agent_keys) + ([] if no_local else list(local_keys)) + [global_keys]
    vals = list(agent_vals) + ([] if no_local else list(local_vals)) + [global_vals]
    if len(keys) != plan.n_streams:
        raise ValueError(f"expected {plan.n_streams} key/value caches, got {len(keys)}")
    ks = [_kv_rows(k, "keys") for k in keys]
    vs = [_kv_rows(v, "values") for v in vals]
    q = roped_q.reshape(s, heads * head_dim)
    if q.stride(-1) != 1 or (q.stride(0) * 2) % 16 or q.data_ptr() % 16:
        q = q.contiguous()
    out = torch.empty((s, heads * head_dim), dtype=torch.bfloat16, device=dev)
    import ctypes
    n = len(ks)
    kp = (ctypes.c_void_p * n)(*[k.data_ptr() for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.data_ptr() for v in vs])
    rows = (ctypes.c_int64 * n)(*[k.shape[0] for k in ks])
    strides = (ctypes.c_int64 * n)(*[k.stride(0) if k.numel() else heads * head_dim for k in ks])
    for k, v in zip(ks, vs):
        if v.shape != k.shape or (v.numel() and v.stride(0) != k.stride(0)):
            raise ValueError("each value cache must match its key cache's shape and layout")
    err = _dev_err(dev)
    lib = _lib.lib()
    st = stream_ptr(dev)
    part = None
    q2 = None
    if plan.q2_src is not None:
        # packed hub rows: a second query block, outputs through the row map
        q2 = q.index_select(0, plan.q2_src)
        part = HierPartialOut()
        part.q2, part.q2_rows, part.q2_stride, part.q2_row0 = (q2.data_ptr(), q2.shape[0],
                                                              q2.stride(0), s)
        part.o, part.o_stride, part.lse, part.row0 = None, 0, None, 0
    chunks = int(os.environ.get(CACHED_SPLIT_ENV, "2"))
    if plan.n_pairs > 0 and chunks > 1:
        # split-KV: partial rows per chunk, then one log-sum-exp merge
        pairs = torch.empty((plan.n_pairs * chunks, 8), dtype=torch.int32, device=dev)
        order = torch.empty(plan.n_pairs * chunks, dtype=torch.int32, device=dev)
        check(lib.hier_plan_split_kv(ptr(plan.q_pairs), plan.n_pairs, chunks, ptr(pairs),
                                     ptr(order), st))
        off, prow, slot = _split_csr(s, plan.q2_src, chunks, dev)
        part_o = torch.empty((chunks * slot, heads * head_dim), dtype=torch.bfloat16, device=dev)
        part_lse = torch.empty((chunks * slot, heads), dtype=torch.float32, device=dev)
        if part is None:
            part = HierPartialOut()
            part.q2, part.q2_rows, part.q2_stride, part.q2_row0 = None, 0, 0, 0
        part.o, part.o_stride, part.lse, part.row0 = (part_o.data_ptr(), part_o.stride(0),
                                                      part_lse.data_ptr(), 0)
        part.slot_rows = slot
        check(lib.hier_attn_fwd_streams(
            ptr(q), s, q.stride(0), n, kp, vp, rows, strides, ptr(out), out.stride(0), None,
            heads, head_dim, ptr(pairs), plan.n_pairs * chunks, ptr(plan.kv_tiles),
            ptr(plan.tile_masks), 1, ptr(order), 1.0 / math.sqrt(head_dim), None,
            ctypes.byref(part), ptr(err), st))
        check(lib.hier_lse_gather_merge(ptr(part_o), part_o.stride(0), ptr(part_lse), heads,
                                        head_dim, ptr(off), ptr(prow), s, ptr(out), out.stride(0),
                                        None, st))
    elif plan.n_pairs > 0:
        check(lib.hier_attn_fwd_streams(
            ptr(q), s, q.stride(0), n, kp, vp, rows, strides, ptr(out), out.stride(0),
            ptr(plan.out_rows), heads, head_dim, ptr(plan.q_pairs), plan.n_pairs,
            ptr(plan.kv_tiles), ptr(plan.tile_masks), 1, ptr(plan.order),
            1.0 / math.sqrt(head_dim), None, None if part is None else ctypes.byref(part),
            ptr(err), st))
    if SYNC_CHECKS if sync_checks is None else sync_checks:
        st = int(plan.status.item())
        if st & 1:
            raise IndexError("list index out of range")
        if st & 2:
            raise RuntimeError("cached attention plan exceeded its tile capacity")
        if int(err.item()):
            raise RuntimeError(f"attention kernel pipeline timeout (code {int(err.item())})")
    return out.reshape(b, s, heads * head_dim)

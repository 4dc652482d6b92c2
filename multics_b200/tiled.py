"""Tiled128 layouts and attention on B200
(``multics/models/kernels/hier_tiled_attention.py``).

* :class:`HierTiledBlockLayout` - the reference's layout record (same fields)
  plus the tcgen05 attention plan built in the same device pass;
* :func:`build_hier_tiled_full_sequence_layouts` (``:244-429``) and
  :func:`build_hier_tiled_cached_layout` (``:474-655``) - bit-exact device
  builders, LRU-cached like the reference
  (``WAN_HIER_TILED_LAYOUT_CACHE_SIZE``, default 2);
* :func:`build_hier_query_active_mask` (``:432-459``);
* :func:`hierarchical_tiled_full_sequence_attention` (``:734-796``) and
  :func:`hierarchical_tiled_cached_attention` (``:658-731``).
"""

from __future__ import annotations

import ctypes
import math
import os
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import HierTiledGrouping, HierTiledSizes, check, ptr, stream_ptr

__all__ = ["HierTiledBlockLayout", "build_hier_tiled_full_sequence_layouts",
           "build_hier_tiled_cached_layout", "build_hier_query_active_mask",
           "hierarchical_tiled_full_sequence_attention", "hierarchical_tiled_cached_attention",
           "clear_hier_tiled_layout_cache", "BLOCK_M", "BLOCK_N"]

BLOCK_M = 16
BLOCK_N = 128
_LAYOUT_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()


class _TiledPlan:
    """Attention plan shared by the layouts of one build (all layouts' pairs)."""

    def __init__(self, q_pairs, kv_tiles, tile_masks, order, n_pairs, pairs_per_layout, status):
        self.q_pairs = q_pairs
        self.kv_tiles = kv_tiles
        self.tile_masks = tile_masks
        self.order = order
        self.n_pairs = n_pairs
        self.pairs_per_layout = pairs_per_layout
        self.status = status


@dataclass(frozen=True)
class HierTiledBlockLayout:
    """Device metadata for one temporal-block launch (reference fields), plus
    the tcgen05 plan of the same segments."""

    prog_qbase: torch.Tensor
    prog_nq: torch.Tensor
    prog_seg: torch.Tensor
    kv_index: torch.Tensor
    kv_valid: torch.Tensor
    kv_count: torch.Tensor
    logical_slots: int
    physical_slots: int
    dense_slots: int
    plan: Optional[_TiledPlan] = field(default=None, compare=False, repr=False)
    plan_layout: int = field(default=0, compare=False, repr=False)


def clear_hier_tiled_layout_cache() -> None:
    _LAYOUT_CACHE.clear()


def _cache_get(key):
    v = _LAYOUT_CACHE.get(key)
    if v is not None:
        _LAYOUT_CACHE.move_to_end(key)
    return v


def _cache_put(key, value):
    limit = max(int(os.environ.get("WAN_HIER_TILED_LAYOUT_CACHE_SIZE", "2")), 0)
    if limit == 0:
        return
    _LAYOUT_CACHE[key] = value
    _LAYOUT_CACHE.move_to_end(key)
    while len(_LAYOUT_CACHE) > limit:
        _LAYOUT_CACHE.popitem(last=False)


def _as_rows(t, dtype):
    cpu = t.detach().to(device="cpu", dtype=dtype)
    if dtype == torch.bool:
        return tuple(tuple(bool(x) for x in r) for r in cpu.tolist())
    return tuple(tuple(int(x) for x in r) for r in cpu.tolist())


def _build_layouts(g: HierTiledGrouping, keep, dev) -> tuple:
    """Count pass, one host read of the counts, fill pass."""
    lib = _lib.lib()
    sz = HierTiledSizes()
    check(lib.hier_tiled_sizes(ctypes.byref(g), ctypes.byref(sz)))
    s = stream_ptr(dev)
    nl, ns = sz.n_layouts, sz.n_seg
    kv_count = torch.zeros(nl * ns, dtype=torch.int32, device=dev)
    n_boxes = torch.zeros(nl * ns, dtype=torch.int32, device=dev)
    slots = torch.zeros((nl * ns, 2), dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib.hier_tiled_count(ctypes.byref(g), ptr(kv_count), ptr(n_boxes), ptr(slots),
                               ptr(status), s))
    counts = kv_count.view(nl, ns).cpu()
    sl = slots.view(nl, ns, 2).cpu()
    if int(status.item()) & 4:
        raise KeyError("a current query frame is missing from an agent cache")
    widths = [max(math.ceil(max(int(counts[b].max()) if ns else 1, 1) / BLOCK_N) * BLOCK_N,
                  BLOCK_N) for b in range(nl)]
    offs = [0]
    for b in range(nl):
        offs.append(offs[-1] + ns * widths[b])
    kv_index = torch.empty(offs[-1], dtype=torch.int32, device=dev)
    kv_valid = torch.empty(offs[-1], dtype=torch.uint8, device=dev)
    kv_off = torch.tensor(offs[:-1], dtype=torch.int64).to(dev)
    kv_w = torch.tensor(widths, dtype=torch.int32).to(dev)
    prog_qbase = torch.empty(nl * sz.n_prog, dtype=torch.int32, device=dev)
    prog_nq = torch.empty_like(prog_qbase)
    prog_seg = torch.empty_like(prog_qbase)
    n_pairs = nl * sz.n_pairs
    cap = max(sz.tile_capacity, 1)
    q_pairs = torch.empty((max(n_pairs, 1), 8), dtype=torch.int32, device=dev)
    kv_tiles = torch.empty((cap, 4), dtype=torch.int32, device=dev)
    tile_masks = torch.empty((cap, 4), dtype=torch.int32, device=dev)
    order = torch.empty(max(n_pairs, 1), dtype=torch.int32, device=dev)
    check(lib.hier_tiled_build(ctypes.byref(g), ptr(n_boxes), ptr(kv_off), ptr(kv_w),
                               ptr(prog_qbase), ptr(prog_nq), ptr(prog_seg), ptr(kv_index),
                               ptr(kv_valid), ptr(q_pairs), ptr(kv_tiles), ptr(tile_masks), cap,
                               ptr(order), ptr(status), s))
    plan = _TiledPlan(q_pairs, kv_tiles, tile_masks, order, n_pairs, sz.n_pairs, status)
    del keep
    out = []
    for b in range(nl):
        cnt = counts[b]
        out.append(HierTiledBlockLayout(
            prog_qbase=prog_qbase[b * sz.n_prog:(b + 1) * sz.n_prog],
            prog_nq=prog_nq[b * sz.n_prog:(b + 1) * sz.n_prog],
            prog_seg=prog_seg[b * sz.n_prog:(b + 1) * sz.n_prog],
            kv_index=kv_index[offs[b]:offs[b + 1]].view(ns, widths[b]),
            kv_valid=kv_valid[offs[b]:offs[b + 1]].view(ns, widths[b]),
            kv_count=kv_count[b * ns:(b + 1) * ns],
            logical_slots=int(sl[b, :, 0].sum()), physical_slots=int(cnt.sum()),
            dense_slots=int(sl[b, :, 1].sum()), plan=plan, plan_layout=b))
    return tuple(out)


def build_hier_tiled_full_sequence_layouts(*, device, num_players: int, num_frames: int,
                                           num_patches: int, num_groups: int,
                                           num_local_hub_tokens: int, num_global_hub_tokens: int,
                                           num_frame_per_block: int, local_attn_size: int,
                                           group_labels: torch.Tensor, active_group: torch.Tensor,
                                           direct_player: bool) -> tuple:
    """Full-sequence metadata equivalent to cached Tiled128 launches."""
    P, T, L = int(num_players), int(num_frames), int(num_patches)
    N, KL, KG = int(num_groups), int(num_local_hub_tokens), int(num_global_hub_tokens)
    n, window = int(num_frame_per_block), int(local_attn_size)
    if T % n != 0:
        raise ValueError(f"Tiled128 requires T % n == 0, got T={T}, n={n}")
    if window != -1 and window < n:
        raise ValueError(f"Tiled128 requires local_attn_size=-1 or >=n, got {window}, n={n}")
    if tuple(group_labels.shape) != (T, P) or tuple(active_group.shape) != (T, N):
        raise ValueError(
            "Tiled128 grouping shape mismatch: "
            f"labels={tuple(group_labels.shape)} expected {(T, P)}, "
            f"active={tuple(active_group.shape)} expected {(T, N)}")
    labels = _as_rows(group_labels, torch.long)
    active = _as_rows(active_group, torch.bool)
    for start in range(0, T, n):
        if any(labels[t] != labels[start] for t in range(start + 1, min(start + n, T))):
            raise ValueError("Tiled128 requires group labels constant inside each temporal block")
    dev = torch.device(device)
    key = (str(dev), P, T, L, N, KL, KG, n, window, labels, active, bool(direct_player), BLOCK_M,
           BLOCK_N)
    hit = _cache_get(key)
    if hit is not None:
        return hit
    if dev.type != "cuda":
        raise NotImplementedError("the B200 Tiled128 builder runs on CUDA devices only")
    lab = torch.tensor(labels, dtype=torch.int64, device=dev).reshape(T, P)
    act = torch.tensor(active, dtype=torch.uint8, device=dev).reshape(T, N)
    g = HierTiledGrouping()
    g.mode = 0
    g.P, g.N, g.L, g.KL, g.KG = P, N, L, KL, KG
    g.n_block, g.local_attn, g.direct, g.T = n, window, int(bool(direct_player)), T
    g.labels, g.active = lab.data_ptr(), act.data_ptr()
    result = _build_layouts(g, (lab, act), dev)
    _cache_put(key, result)
    return result


def build_hier_tiled_cached_layout(*, device, P: int, N: int, L: int, KL: int, KG: int,
                                   n_frames: int, n_block: int, local_attn: int,
                                   agent_frame_lists: Sequence[Sequence[int]],
                                   local_frame_lists: Sequence[Sequence[int]],
                                   global_frame_list: Sequence[int],
                                   local_active_frames: Sequence[Sequence[bool]],
                                   labels: Sequence[Sequence[int]],
                                   q_active: Sequence[Sequence[bool]],
                                   direct_player: bool) -> HierTiledBlockLayout:
    """Metadata from the live cached-inference frame lists."""
    if not agent_frame_lists or any(len(x) != len(agent_frame_lists[0]) for x in agent_frame_lists):
        raise ValueError("Tiled128 requires equal agent cache lengths")
    if not local_frame_lists or any(len(x) != len(local_frame_lists[0]) for x in local_frame_lists):
        raise ValueError("Tiled128 requires equal local cache lengths")
    af = tuple(tuple(int(x) for x in r) for r in agent_frame_lists)
    lf = tuple(tuple(int(x) for x in r) for r in local_frame_lists)
    gf = tuple(int(x) for x in global_frame_list)
    la = tuple(tuple(bool(x) for x in r) for r in local_active_frames)
    lab_t = tuple(tuple(int(x) for x in r) for r in labels)
    qa_t = tuple(tuple(bool(x) for x in r) for r in q_active)
    dev = torch.device(device)
    key = ("cached", str(dev), P, N, L, KL, KG, n_frames, n_block, local_attn, af, lf, gf, la,
           lab_t, qa_t, bool(direct_player), BLOCK_M, BLOCK_N)
    hit = _cache_get(key)
    if hit is not None:
        return hit[0]
    qf = gf[-n_frames:] if KG > 0 else af[0][-n_frames:]
    if len(qf) != n_frames:
        raise ValueError("Tiled128 cannot identify the current cached query frames")
    for p in range(P):
        missing = [f for f in qf if f not in af[p]]
        if missing:
            raise KeyError(missing[0])
    if dev.type != "cuda":
        raise NotImplementedError("the B200 Tiled128 builder runs on CUDA devices only")

    def frames(fr, w):
        return torch.tensor(list(fr), dtype=torch.int64).repeat_interleave(max(w, 1)).to(dev)

    agent = [frames(f, L) for f in af]
    local = [frames(f, KL) for f in lf]
    lact = [torch.tensor(list(a), dtype=torch.uint8).repeat_interleave(max(KL, 1)).to(dev)
            for a in la]
    glob = frames(gf, KG) if KG > 0 else None
    lab = torch.tensor(lab_t, dtype=torch.int64, device=dev).reshape(n_frames, P)
    qact = torch.tensor(qa_t, dtype=torch.uint8, device=dev).reshape(n_frames, N)
    g = HierTiledGrouping()
    g.mode = 1
    g.P, g.N, g.L, g.KL, g.KG = P, N, L, KL, KG
    g.n_block, g.local_attn, g.direct = n_block, local_attn, int(bool(direct_player))
    g.n_frames, g.fa, g.fl, g.fg = n_frames, len(af[0]), len(lf[0]), len(gf) if KG > 0 else 0
    g.labels, g.active = lab.data_ptr(), qact.data_ptr()
    for i, t in enumerate(agent):
        g.agent_frames[i] = t.data_ptr()
    for i, t in enumerate(local):
        g.local_frames[i] = t.data_ptr()
    for i, t in enumerate(lact):
        g.local_active[i] = t.data_ptr()
    g.global_frames = glob.data_ptr() if glob is not None else None
    result = _build_layouts(g, (agent, local, lact, glob, lab, qact), dev)
    _cache_put(key, result)
    return result[0]


def build_hier_query_active_mask(*, active_group, num_players, num_frames, num_patches,
                                 num_groups, num_local_hub_tokens, num_global_hub_tokens, device,
                                 dtype) -> torch.Tensor:
    """``[1,S,1]`` row mask: only inactive local-hub query rows are zero."""
    P, T, L = int(num_players), int(num_frames), int(num_patches)
    N, KL, KG = int(num_groups), int(num_local_hub_tokens), int(num_global_hub_tokens)
    if tuple(active_group.shape) != (T, N):
        raise ValueError(f"active_group must have shape {(T, N)}, got {tuple(active_group.shape)}")
    agent = torch.ones(P * T * L, device=device, dtype=dtype)
    local = active_group.to(device=device, dtype=dtype).reshape(T, N, 1).expand(T, N, KL).reshape(-1)
    glob = torch.ones(T * KG, device=device, dtype=dtype)
    return torch.cat((agent, local, glob), dim=0).view(1, -1, 1)


def hierarchical_tiled_full_sequence_attention(*, roped_q: torch.Tensor, roped_k: torch.Tensor,
                                               value: torch.Tensor,
                                               layouts: Sequence[HierTiledBlockLayout]):
    """Forward over projected full-sequence Q/K/V with layouts from this module."""
    if roped_k.shape != value.shape or roped_q.ndim != 4 or roped_k.ndim != 4:
        raise ValueError(
            f"Tiled128 expects Q [B,Sq,H,D] and matching K/V [B,Sk,H,D], "
            f"got {roped_q.shape}, {roped_k.shape}, {value.shape}")
    batch, seq_len, heads, head_dim = roped_q.shape
    if roped_k.shape[0] != batch or roped_k.shape[2:] != (heads, head_dim):
        raise ValueError(
            f"Tiled128 Q/K batch/head shapes must match, got {roped_q.shape}, {roped_k.shape}")
    if batch != 1 or head_dim != 128 or roped_q.dtype != torch.bfloat16:
        raise NotImplementedError(
            "Tiled128 training currently supports B=1, BF16, head_dim=128; "
            f"got B={batch}, dtype={roped_q.dtype}, head_dim={head_dim}")
    if not roped_q.is_cuda:
        raise NotImplementedError("Tiled128 training requires CUDA")
    if roped_k.dtype != roped_q.dtype or value.dtype != roped_q.dtype:
        raise ValueError("Tiled128 Q/K/V dtypes must match")
    q = roped_q.reshape(seq_len, heads * head_dim)
    k = roped_k.reshape(-1, heads * head_dim)
    v = value.reshape(-1, heads * head_dim)
    q, k, v = (t if t.is_contiguous() else t.contiguous() for t in (q, k, v))
    out = torch.zeros_like(q)
    groups = OrderedDict()
    for lay in layouts:
        if lay.plan is None:
            raise TypeError("layouts must come from multics_b200.tiled builders")
        groups.setdefault(id(lay.plan), (lay.plan, []))[1].append(lay.plan_layout)
    from .attention import _dev_err
    err = _dev_err(q.device)
    lib = _lib.lib()
    for plan, idx in groups.values():
        per = plan.pairs_per_layout
        full = sorted(idx) == list(range(plan.n_pairs // max(per, 1))) and len(set(idx)) == len(idx)
        if full:
            ranges = [(0, plan.n_pairs, plan.order)]
        else:
            ranges = [(b * per, (b + 1) * per, None) for b in sorted(set(idx))]
        for p0, p1, order in ranges:
            if p1 <= p0:
                continue
            kp = (ctypes.c_void_p * 1)(k.data_ptr())
            vp = (ctypes.c_void_p * 1)(v.data_ptr())
            rows = (ctypes.c_int64 * 1)(k.shape[0])
            strides = (ctypes.c_int64 * 1)(k.stride(0))
            qp = plan.q_pairs[p0:p1]
            check(lib.hier_attn_fwd_streams(
                ptr(q), seq_len, q.stride(0), 1, kp, vp, rows, strides, ptr(out), out.stride(0),
                None, heads, head_dim, ptr(qp), p1 - p0, ptr(plan.kv_tiles), ptr(plan.tile_masks), 1,
                ptr(order), 1.0 / math.sqrt(head_dim), None, None, ptr(err), stream_ptr(q.device)))
    return out.reshape(batch, seq_len, heads * head_dim)


def hierarchical_tiled_cached_attention(*, roped_q, agent_frames, agent_keys, agent_vals,
                                        local_frames, local_keys, local_vals, local_active_tokens,
                                        global_frames, global_keys, global_vals, labels, active, P,
                                        N, L, KL, KG, n_frames, n_block, local_attn,
                                        direct_player):
    """Cached-inference Tiled128 plugin: the same logical edges as the
    cached backends, run in place over the rolling caches."""
    b, seq_len, heads, head_dim = roped_q.shape
    if b != 1 or head_dim != 128 or roped_q.dtype != torch.bfloat16:
        raise NotImplementedError(
            "cached Tiled128 supports B=1, BF16, head_dim=128; "
            f"got B={b}, dtype={roped_q.dtype}, head_dim={head_dim}")
    if not roped_q.is_cuda:
        raise NotImplementedError("cached Tiled128 requires CUDA")
    from .cached import hierarchical_cached_attention
    return hierarchical_cached_attention(
        roped_q=roped_q, agent_frames=agent_frames, agent_keys=agent_keys, agent_vals=agent_vals,
        local_frames=local_frames, local_keys=local_keys, local_vals=local_vals,
        local_active_tokens=local_active_tokens, global_frames=global_frames,
        global_keys=global_keys, global_vals=global_vals, labels=labels, active=active, P=P, N=N,
        L=L, KL=KL, KG=KG, n_frames=n_frames, n_block=n_block, local_attn=local_attn,
        direct_player=direct_player)

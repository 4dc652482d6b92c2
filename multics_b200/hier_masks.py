"""Hierarchical masks and block plans, built on the GPU.

Mirrors the public API of the reference's ``multics/models/hier_masks.py``
(same function names, argument meaning and error messages) with the mask
predicate evaluated by CUDA kernels of ``libhier_b200.so``:

* ``build_stage2_hier_self_attn_mask`` (``hier_masks.py:364-641``) returns the
  dense ``[S,S]`` bool mask from ``hier_dense_mask``;
* ``build_stage2_hier_flex_block_mask`` (``hier_masks.py:722-1149``) returns a
  :class:`HierBlockMask` - the Flex BlockMask block lists plus the attention
  work plan (query tiles, key tiles, per-row key bitmasks of partial blocks)
  consumed by the tcgen05 attention kernel - together with ``S`` and
  ``S_pad`` like the reference.
"""

from __future__ import annotations

import ctypes
import math
import os
from collections import OrderedDict
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import HierGrouping, check, ptr, stream_ptr

_HIER_LOCAL_HUB_MODES = ("shared", "per_group")
_BLOCK_PLAN_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()


# ---------------------------------------------------------------------------
# grouping normalisation (host side, reference messages)
# ---------------------------------------------------------------------------


def _prepare_hier_group_tensors(group_labels, active_group, num_players, num_frames,
                                num_groups, device):
    """Normalise labels/active (``hier_masks.py:22-71``): labels ``[T,P]`` in
    ``[0,N)``, active ``[T,N]`` (scatter of labels when not given)."""
    if group_labels is None:
        raise ValueError("hier_hub requires group_labels [T,P] or [1,T,P]")
    labels = group_labels
    if labels.dim() == 3:
        if labels.shape[0] != 1:
            raise ValueError(f"hier_hub expects group_labels batch B=1, got {tuple(labels.shape)}")
        labels = labels[0]
    if labels.shape != (num_frames, num_players):
        raise ValueError(
            f"group_labels must be [T={num_frames},P={num_players}], got {tuple(labels.shape)}")
    labels = labels.to(device=device, dtype=torch.long).contiguous()
    if labels.numel():
        lo, hi = (int(x) for x in torch.stack([labels.min(), labels.max()]).tolist())
        if lo < 0 or hi >= num_groups:
            raise ValueError(
                f"group_labels values must be in [0,{num_groups}), got min={lo} max={hi}")
    if active_group is None:
        active = torch.zeros(num_frames, num_groups, device=device, dtype=torch.bool)
        active.scatter_(1, labels, True)
    else:
        active = active_group
        if active.dim() == 3:
            if active.shape[0] != 1:
                raise ValueError(
                    f"hier_hub expects active_group batch B=1, got {tuple(active.shape)}")
            active = active[0]
        if active.shape != (num_frames, num_groups):
            raise ValueError(
                f"active_group must be [T={num_frames},N={num_groups}], got {tuple(active.shape)}")
        active = active.to(device=device, dtype=torch.bool).contiguous()
    return labels, active


def _squeeze_hier_batch(tensor, expected_tail_ndim, name):
    """Drop an optional leading B=1 dim (``hier_masks.py:74-91``)."""
    if tensor.dim() == expected_tail_ndim + 1:
        if tensor.shape[0] != 1:
            raise ValueError(f"{name} batch B must be 1, got {tuple(tensor.shape)}")
        tensor = tensor[0]
    if tensor.dim() != expected_tail_ndim:
        raise ValueError(
            f"{name} must have rank {expected_tail_ndim} or {expected_tail_ndim + 1} with B=1, got {tuple(tensor.shape)}")
    return tensor


def _slice_hier_active_group_for_cached_mask(active_group, start_frame, num_frames):
    """Current-block slice of a full-clip active tensor (``hier_masks.py:101-124``)."""
    if active_group is None:
        return None
    active = _squeeze_hier_batch(active_group, 2, "active_group")
    start, n = int(start_frame), int(num_frames)
    if start < 0 or n <= 0:
        raise ValueError(f"invalid cached active_group slice: start={start}, n={n}")
    if active.shape[0] == n:
        return active.contiguous()
    if start + n > active.shape[0]:
        raise ValueError(
            f"active_group T={active.shape[0]} does not cover cached block [{start},{start + n})")
    return active[start:start + n].contiguous()


def _prepare_hier_membership_tensors(membership, global_only, active_group, num_players,
                                     num_frames, num_groups, device, *, allow_full_t=False):
    """Normalise membership/global_only/active (``hier_masks.py:127-193``)."""
    if membership is None:
        raise ValueError("hier_group_format=membership requires membership [T,N,P] or [1,T,N,P]")
    mem = _squeeze_hier_batch(membership, 3, "membership")
    T, N, P = (int(mem.shape[0]), int(mem.shape[1]), int(mem.shape[2]))
    if P != num_players:
        raise ValueError(
            f"membership P={P} must equal num_players={num_players}, got {tuple(mem.shape)}")
    if N != num_groups:
        raise ValueError(
            f"membership N={N} must equal num_groups={num_groups}, got {tuple(mem.shape)}")
    if num_frames is not None:
        if allow_full_t:
            if T < int(num_frames):
                raise ValueError(f"membership T={T} shorter than current block n={int(num_frames)}")
        elif T != int(num_frames):
            raise ValueError(
                f"membership must be [T={int(num_frames)},N={num_groups},P={num_players}], got {tuple(mem.shape)}")
    mem = mem.to(device=device, dtype=torch.bool).contiguous()
    if global_only is None:
        raise ValueError("hier_group_format=membership requires global_only [T,P] or [1,T,P]")
    go = _squeeze_hier_batch(global_only, 2, "global_only")
    if go.shape != (T, P):
        raise ValueError(f"global_only must be [T={T},P={P}], got {tuple(go.shape)}")
    go = go.to(device=device, dtype=torch.bool).contiguous()
    if active_group is None:
        active = mem.any(dim=-1)
    else:
        active = _squeeze_hier_batch(active_group, 2, "active_group")
        if allow_full_t and active.shape != (T, N):
            active = mem.any(dim=-1).contiguous()
        elif active.shape != (T, N):
            raise ValueError(f"active_group must be [T={T},N={N}], got {tuple(active.shape)}")
        else:
            active = active.to(device=device, dtype=torch.bool).contiguous()
    return mem, go, active


def _refuse_membership_on_scalar_kernel(*, attn_impl=None, infer_kernel=None):
    """Reference fail-fast for scalar-label kernels (``hier_masks.py:196-207``)."""
    if attn_impl == "hier_tiled_ste":
        raise ValueError(
            "hier_group_format=membership is not supported with attn_impl=hier_tiled_ste; use --attn_impl flex or sdpa until the kernel grows a membership lookup")
    if infer_kernel in ("segmented", "tiled128"):
        raise ValueError(
            f"hier_group_format=membership is not supported with WAN_HIER_INFER_KERNEL={infer_kernel}; use sdpa (or full_sequence flex)")


def _validate_hier_no_local_topology(no_local, KL, KG):
    """``hier_masks.py:210-214``."""
    if bool(no_local) and (int(KL) != 0 or int(KG) <= 0):
        raise ValueError(f"hier_no_local_hub requires K_L=0 and K_G>0; got K_L={KL}, K_G={KG}")


def normalize_hier_local_hub_mode(mode):
    """``hier_masks.py:217-223``."""
    mode = str(mode).strip().lower()
    if mode not in _HIER_LOCAL_HUB_MODES:
        raise ValueError(f"hier_local_hub_mode must be shared or per_group; got {mode!r}")
    return mode


# ---------------------------------------------------------------------------
# grouping spec shared by the CUDA builders
# ---------------------------------------------------------------------------


@dataclass
class HierGroupingSpec:
    """Validated grouping tensors (device) + dims, convertible to the C struct."""

    P: int
    T: int
    L: int
    N: int
    KL: int
    KG: int
    n_block: int
    local_attn: int
    direct: bool
    no_local: bool
    labels: Optional[torch.Tensor]
    membership: Optional[torch.Tensor]
    global_only: Optional[torch.Tensor]
    active: torch.Tensor

    @property
    def S(self) -> int:
        return self.P * self.T * self.L + self.T * (self.N * self.KL + self.KG)

    @property
    def membership_mode(self) -> bool:
        return self.membership is not None

    def c_struct(self) -> HierGrouping:
        g = HierGrouping()
        g.P, g.T, g.L, g.N, g.KL, g.KG = self.P, self.T, self.L, self.N, self.KL, self.KG
        g.n_block, g.local_attn = self.n_block, self.local_attn
        g.direct, g.no_local = int(self.direct), int(self.no_local)
        g.membership_mode = int(self.membership_mode)
        self._u8 = {}
        for name in ("membership", "global_only", "active"):
            t = getattr(self, name)
            if t is not None:
                self._u8[name] = t.to(torch.uint8).contiguous()
        g.labels = self.labels.data_ptr() if self.labels is not None else None
        g.membership = self._u8["membership"].data_ptr() if "membership" in self._u8 else None
        g.global_only = self._u8["global_only"].data_ptr() if "global_only" in self._u8 else None
        g.active = self._u8["active"].data_ptr()
        return g

    def key(self):
        def raw(t):
            return None if t is None else (tuple(t.shape), t.detach().cpu().numpy().tobytes())

        return (self.P, self.T, self.L, self.N, self.KL, self.KG, self.n_block, self.local_attn,
                self.direct, self.no_local, raw(self.labels), raw(self.membership),
                raw(self.global_only), raw(self.active), str(self.active.device))


def make_grouping_spec(num_players, num_frames, num_patches, num_groups, num_local_hub_tokens,
                       num_global_hub_tokens, num_frame_per_block, local_attn_size, group_labels,
                       active_group=None, direct_player=False, device=None, membership=None,
                       global_only=None, hier_no_local_hub=False) -> HierGroupingSpec:
    """Validate like the reference mask builders (``hier_masks.py:408-417,
    537-548``) and return a device-resident grouping spec."""
    P, T, L = int(num_players), int(num_frames), int(num_patches)
    N, KL, KG = int(num_groups), int(num_local_hub_tokens), int(num_global_hub_tokens)
    _validate_hier_no_local_topology(hier_no_local_hub, KL, KG)
    if local_attn_size != -1 and local_attn_size < num_frame_per_block:
        raise ValueError(
            f"hier_hub requires local_attn_size=-1 or >= num_frame_per_block; got local_attn_size={local_attn_size}, n={num_frame_per_block}")
    if device is None:
        device = torch.device("cuda")
    device = torch.device(device)
    if device.type != "cuda":
        raise NotImplementedError(
            "the B200 hierarchical mask builders run on CUDA devices only; got " + str(device))
    if membership is not None:
        if N > 62:
            raise ValueError(f"membership bitset path supports N<=62, got N={N}")
        mem, go, active = _prepare_hier_membership_tensors(
            membership, global_only, active_group, P, T, N, device)
        labels = None
    else:
        labels, active = _prepare_hier_group_tensors(group_labels, active_group, P, T, N, device)
        mem = go = None
    return HierGroupingSpec(P, T, L, N, KL, KG, int(num_frame_per_block), int(local_attn_size),
                            bool(direct_player), bool(hier_no_local_hub), labels, mem, go, active)


# ---------------------------------------------------------------------------
# dense mask
# ---------------------------------------------------------------------------


def build_stage2_hier_self_attn_mask(num_players, num_frames, num_patches, num_groups,
                                     num_local_hub_tokens, num_global_hub_tokens,
                                     num_frame_per_block, local_attn_size, group_labels,
                                     active_group=None, direct_player=False, device=None,
                                     membership=None, global_only=None,
                                     hier_no_local_hub=False) -> torch.Tensor:
    """Dense ``[S,S]`` bool hierarchical mask (``hier_masks.py:364-641``),
    computed by the ``hier_dense_mask`` CUDA kernel.  Bit-exact with the
    reference."""
    spec = make_grouping_spec(num_players, num_frames, num_patches, num_groups,
                              num_local_hub_tokens, num_global_hub_tokens, num_frame_per_block,
                              local_attn_size, group_labels, active_group, direct_player, device,
                              membership, global_only, hier_no_local_hub)
    return HierDenseMask.wrap(dense_mask_rows(spec, 0, spec.S), spec)


class HierDenseMask(torch.Tensor):
    """The dense ``[S,S]`` bool mask of :func:`build_stage2_hier_self_attn_mask`
    (a plain bool tensor for every torch operation, whose results are plain
    tensors) that also carries the grouping it was built from, so that
    :class:`multics_b200.attention.SelfAttention` runs it on the grouping's
    work plan instead of reading the mask's bytes."""

    hier_spec: "HierGroupingSpec"

    __torch_function__ = torch._C._disabled_torch_function_impl

    @staticmethod
    def wrap(mask: torch.Tensor, spec: "HierGroupingSpec") -> "HierDenseMask":
        m = mask.as_subclass(HierDenseMask)
        m.hier_spec = spec
        return m


def dense_mask_rows(spec: HierGroupingSpec, row0: int, nrows: int) -> torch.Tensor:
    out = torch.empty(nrows, spec.S, dtype=torch.bool, device=spec.active.device)
    g = spec.c_struct()
    check(_lib.lib().hier_dense_mask(ctypes.byref(g), row0, nrows, ptr(out), stream_ptr()))
    return out


# ---------------------------------------------------------------------------
# block mask + attention plan
# ---------------------------------------------------------------------------


@dataclass
class HierBlockMask:
    """Block-sparse description of the hierarchical mask at 128x128 blocks.

    ``kv_num_blocks / kv_indices / full_kv_num_blocks / full_kv_indices`` have
    the shapes of the Flex BlockMask fields (``[1,1,nb]`` / ``[1,1,nb,nb]``)
    with the same values in each row's valid prefix.  ``q_pairs``,
    ``kv_tiles``, ``row_masks`` and ``order`` are the attention work plan
    (see include/hier_b200.h, hier_block_plan_build)."""

    S: int
    S_pad: int
    kv_num_blocks: torch.Tensor
    kv_indices: torch.Tensor
    full_kv_num_blocks: torch.Tensor
    full_kv_indices: torch.Tensor
    kv_offsets: torch.Tensor
    full_offsets: torch.Tensor
    kv_flat: torch.Tensor
    full_flat: torch.Tensor
    q_pairs: torch.Tensor
    kv_tiles: torch.Tensor
    row_masks: torch.Tensor
    order: torch.Tensor
    n_partial: int
    n_full: int
    n_kv_tiles: torch.Tensor
    spec: Optional[HierGroupingSpec]

    @property
    def shape(self):
        return (1, 1, self.S_pad, self.S_pad)

    @property
    def num_pairs(self) -> int:
        return self.q_pairs.shape[0]

    def tile_flops(self, head_dim: int, heads: int) -> float:
        """FLOPs of all computed 128x128 tiles (full + partial), 4*128*128*D each."""
        return 4.0 * 128 * 128 * head_dim * heads * (self.n_partial + self.n_full)


def build_block_plan(spec: HierGroupingSpec, page_table: Optional[torch.Tensor] = None) -> HierBlockMask:
    """Run the CUDA block classifier + plan builder for ``spec``.

    One host synchronisation reads the number of partial blocks to size the
    row-mask table (the reference reads its grouping to the host as well)."""
    dev = spec.active.device
    S = spec.S
    nb = (S + 127) // 128
    L = _lib.lib()
    g = spec.c_struct()
    ws_bytes = ctypes.c_size_t()
    check(L.hier_block_workspace_size(ctypes.byref(g), ctypes.byref(ws_bytes)))
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    kv_num = torch.empty(nb, **i32)
    full_num = torch.empty(nb, **i32)
    kv_off = torch.empty(nb + 1, **i32)
    full_off = torch.empty(nb + 1, **i32)
    kv_flat = torch.empty(nb * nb, **i32)
    full_flat = torch.empty(nb * nb, **i32)
    totals = torch.zeros(2, **i32)
    s = stream_ptr()
    check(L.hier_block_mask_build(ctypes.byref(g), ptr(ws), ptr(kv_num), ptr(kv_off), ptr(kv_flat),
                                  ptr(full_num), ptr(full_off), ptr(full_flat), ptr(totals), s))
    n_partial, n_full = (int(x) for x in totals.tolist())
    n_pairs = (nb + 1) // 2
    q_pairs = torch.empty(n_pairs, 8, **i32)
    kv_tiles = torch.empty(max(n_partial + n_full, 1), 4, **i32)
    row_masks = torch.empty(max(n_partial, 1), 128, 4, **i32)
    order = torch.empty(n_pairs, **i32)
    n_kv_tiles = torch.zeros(1, **i32)
    if page_table is not None:
        pt = page_table.to(device=dev, dtype=torch.int32).contiguous()
        need = 2 * nb
        if pt.numel() < need:
            pt = torch.cat([pt, pt.new_zeros(need - pt.numel())])
    else:
        pt = None
    check(L.hier_block_plan_build(ctypes.byref(g), ptr(ws), ptr(kv_off), ptr(kv_flat),
                                  ptr(full_off), ptr(full_flat), ptr(pt), ptr(q_pairs),
                                  ptr(kv_tiles), ptr(row_masks), ptr(order), ptr(n_kv_tiles), s))
    return _block_mask_from_lists(S, nb, kv_num, kv_off, kv_flat[:n_partial], full_num,
                                  full_off, full_flat[:n_full], q_pairs, kv_tiles, row_masks,
                                  order, n_partial, n_full, n_kv_tiles, spec)


def _block_mask_from_lists(S, nb, kv_num, kv_off, kv_flat, full_num, full_off, full_flat,
                           q_pairs, kv_tiles, row_masks, order, n_partial, n_full, n_kv_tiles,
                           spec) -> HierBlockMask:
    dev = kv_num.device

    def padded(flat, off, num):
        # Flex-shaped [1,1,nb,nb] index tensor holding each row's list as prefix
        out = torch.zeros(nb, nb, dtype=torch.int32, device=dev)
        if flat.numel():
            rows = torch.repeat_interleave(torch.arange(nb, device=dev), num.long())
            cols = torch.arange(flat.numel(), device=dev) - off[:-1].long()[rows]
            out[rows, cols] = flat
        return out.view(1, 1, nb, nb)

    return HierBlockMask(
        S=S, S_pad=nb * 128, kv_num_blocks=kv_num.view(1, 1, nb),
        kv_indices=padded(kv_flat, kv_off, kv_num), full_kv_num_blocks=full_num.view(1, 1, nb),
        full_kv_indices=padded(full_flat, full_off, full_num), kv_offsets=kv_off,
        full_offsets=full_off, kv_flat=kv_flat, full_flat=full_flat, q_pairs=q_pairs,
        kv_tiles=kv_tiles, row_masks=row_masks, order=order, n_partial=n_partial,
        n_full=n_full, n_kv_tiles=n_kv_tiles, spec=spec)


def build_dense_block_plan(mask: Optional[torch.Tensor], S: int, device=None) -> HierBlockMask:
    """128x128 block plan of a caller's dense mask (``[S,S]``, or with leading
    unit dims; any non-zero element allows the pair, as ``flash_attention``'s
    ``mask.to(bool)`` does, ``attention.py:47-54``) or of no mask (``None``:
    every pair allowed).  The returned :class:`HierBlockMask` has no grouping
    (``spec`` is None), so it always runs on the block plan."""
    if mask is not None:
        m = mask
        while m.dim() > 2:
            if m.shape[0] != 1:
                raise NotImplementedError(
                    f"the B200 attention takes one [S,S] mask for all batches and heads; got "
                    f"{tuple(mask.shape)}")
            m = m[0]
        if tuple(m.shape) != (S, S):
            raise ValueError(f"mask must be [S={S},S={S}], got {tuple(mask.shape)}")
        if m.dtype != torch.bool and m.dtype != torch.uint8:
            m = m.to(torch.bool)
        dev = m.device if device is None else torch.device(device)
        m = m.to(dev)
        if m.stride(1) != 1:
            m = m.contiguous()
        ld = m.stride(0)
    else:
        dev = torch.device("cuda") if device is None else torch.device(device)
        m, ld = None, S
    nb = (S + 127) // 128
    L = _lib.lib()
    ws_bytes = ctypes.c_size_t()
    check(L.hier_dense_block_workspace_size(S, ctypes.byref(ws_bytes)))
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    kv_num, full_num = torch.empty(nb, **i32), torch.empty(nb, **i32)
    kv_off, full_off = torch.empty(nb + 1, **i32), torch.empty(nb + 1, **i32)
    kv_flat, full_flat = torch.empty(nb * nb, **i32), torch.empty(nb * nb, **i32)
    totals = torch.zeros(2, **i32)
    s = stream_ptr(dev)
    check(L.hier_dense_block_mask_build(ptr(m), S, ld, ptr(ws), ptr(kv_num), ptr(kv_off),
                                        ptr(kv_flat), ptr(full_num), ptr(full_off),
                                        ptr(full_flat), ptr(totals), s))
    n_partial, n_full = (int(x) for x in totals.tolist())
    n_pairs = (nb + 1) // 2
    q_pairs = torch.empty(n_pairs, 8, **i32)
    kv_tiles = torch.empty(max(n_partial + n_full, 1), 4, **i32)
    row_masks = torch.empty(max(n_partial, 1), 128, 4, **i32)
    order = torch.empty(n_pairs, **i32)
    n_kv_tiles = torch.zeros(1, **i32)
    check(L.hier_dense_block_plan_build(ptr(m), S, ld, ptr(ws), ptr(kv_off), ptr(kv_flat),
                                        ptr(q_pairs), ptr(kv_tiles), ptr(row_masks), ptr(order),
                                        ptr(n_kv_tiles), s))
    return _block_mask_from_lists(S, nb, kv_num, kv_off, kv_flat[:n_partial], full_num,
                                  full_off, full_flat[:n_full], q_pairs, kv_tiles, row_masks,
                                  order, n_partial, n_full, n_kv_tiles, None)


def _cache_size():
    return int(os.environ.get("WAN_HIER_BLOCKMASK_CACHE_SIZE", "2"))


def build_stage2_hier_flex_block_mask(num_players, num_frames, num_patches, num_groups,
                                      num_local_hub_tokens, num_global_hub_tokens,
                                      num_frame_per_block, local_attn_size, group_labels,
                                      active_group, direct_player, device, membership=None,
                                      global_only=None, hier_no_local_hub=False):
    """Block mask for the hierarchical semantics (``hier_masks.py:722-1149``).

    Returns ``(HierBlockMask, S, S_pad)``.  Results are cached by grouping
    value with the reference's bounded retention
    (``WAN_HIER_BLOCKMASK_CACHE_SIZE``, default 2, ``hier_masks.py:644-666``)."""
    spec = make_grouping_spec(num_players, num_frames, num_patches, num_groups,
                              num_local_hub_tokens, num_global_hub_tokens, num_frame_per_block,
                              local_attn_size, group_labels, active_group, direct_player, device,
                              membership, global_only, hier_no_local_hub)
    bm = block_mask_for_spec(spec)
    return bm, bm.S, bm.S_pad


def block_mask_for_spec(spec: HierGroupingSpec) -> HierBlockMask:
    """The :class:`HierBlockMask` of a grouping, from the cache of
    :func:`build_stage2_hier_flex_block_mask` (keyed by grouping value)."""
    key = ("hier",) + spec.key()
    hit = _BLOCK_PLAN_CACHE.get(key)
    if hit is not None:
        _BLOCK_PLAN_CACHE.move_to_end(key)
        return hit[0]
    bm = build_block_plan(spec)
    limit = _cache_size()
    if limit != 0:
        _BLOCK_PLAN_CACHE[key] = (bm, bm.S, bm.S_pad)
        while limit > 0 and len(_BLOCK_PLAN_CACHE) > limit:
            _BLOCK_PLAN_CACHE.popitem(last=False)
    return bm


def clear_block_mask_cache():
    _BLOCK_PLAN_CACHE.clear()

"""Hierarchical self-attention on B200: fused prologue + tcgen05 attention.

Drop-in counterparts of the reference's ``multics/models/attention.py``:

* :func:`hier_prep_qk` - camera Q/K add + RMSNorm + RoPE
  (``attention.py:307-365``, ``rope.py:248-254``) in one CUDA kernel;
* :func:`hier_block_attention` - attention over a :class:`HierBlockMask`
  (the role of ``flash_attention(mask)`` / FlexAttention,
  ``attention.py:39-54,322-353``);
* :class:`HierSequencePlan` - the faster work plan the layer entry points
  use for labels groupings: one query pair per player frame over its exact
  key runs, hub queries in 128-row tiles of one group;
* :class:`SelfAttention` - same constructor and ``forward(x, freqs, mask,
  cam_tokens)`` signature as the reference module (``attention.py:255-442``).
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Optional

import numpy as np
import torch
import torch.nn as nn

from . import _lib
from ._lib import check, ptr, stream_ptr
from .hier_masks import HierBlockMask, block_mask_for_spec, build_dense_block_plan

__all__ = ["hier_prep_qk", "hier_block_attention", "freqs_table", "RMSNorm", "SelfAttention",
           "AttentionPlan", "attention_from_plan", "HierSequencePlan", "sequence_plan",
           "hier_attention_layer", "attention_mask_plan", "CrossAttention"]

# Work plan of the full-sequence layer entry points: "segments" (the
# HierSequencePlan wherever the grouping allows it) or "blocks" (always the
# 128x128 block plan of the HierBlockMask).
FULL_SEQUENCE_PLAN_ENV = "MULTICS_B200_FULL_SEQUENCE_PLAN"

_DEV_ERR = {}


def _dev_err(device):
    key = torch.device(device).index
    t = _DEV_ERR.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _DEV_ERR[key] = t
    return t


def device_error(device=None) -> int:
    """Sticky device error word of the attention kernels (0 = no timeout)."""
    dev = torch.device("cuda") if device is None else torch.device(device)
    return int(_dev_err(dev).item())


def freqs_table(freqs: torch.Tensor) -> torch.Tensor:
    """Complex RoPE multipliers ``[S,1,D/2]`` (or ``[S,D/2]``) -> float32
    ``[S, D/2, 2]`` (cos, sin) table read by the prologue kernel."""
    if torch.is_complex(freqs):
        f = torch.view_as_real(freqs.reshape(freqs.shape[0], -1))
    else:
        if freqs.shape[-1] != 2:
            raise ValueError(f"real RoPE tables must end in (cos, sin) pairs, got {tuple(freqs.shape)}")
        f = freqs.reshape(freqs.shape[0], -1, 2)
    return f.to(torch.float32).contiguous()


def _rows(x):
    """View a [B=1,S,C] or [S,C] tensor as [S,C] with unit inner stride."""
    if x.dim() == 3:
        if x.shape[0] != 1:
            raise NotImplementedError(
                f"hierarchical B200 attention supports batch B=1; got B={x.shape[0]}")
        x = x[0]
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def hier_prep_qk(qx, kx, freqs, num_heads, *, norm_q_weight, norm_k_weight, cam_tokens=None,
                 cam_q_weight=None, cam_k_weight=None, eps=1e-6, out=None, out_rows=None,
                 k_out_rows=None):
    """``q = rope(rmsnorm(qx + cam @ Wq^T) * wq)`` and the same for k, bf16.

    ``freqs``: complex ``[S,1,D/2]`` (as built by the reference's freq
    builders) or a float32 ``[S,D/2,2]`` table from :func:`freqs_table`.
    ``out_rows`` (int32 ``[S]`` on the device) writes token ``r`` to row
    ``out_rows[r]`` of the outputs; ``k_out_rows`` gives k its own rows (a
    paged key pool), ``out`` then holds ``(q_out, k_out)`` sized for them."""
    q2, k2 = _rows(qx), _rows(kx)
    S, dim = q2.shape
    if q2.dtype != torch.bfloat16 or k2.dtype != torch.bfloat16:
        raise NotImplementedError("hier_prep_qk expects bf16 q/k projections")
    if k2.shape != q2.shape or k2.stride(0) != q2.stride(0):
        k2 = k2.contiguous()
        q2 = q2.contiguous()
    D = dim // num_heads
    ft = freqs if (freqs.dtype == torch.float32 and freqs.dim() == 3
                   and freqs.shape[-1] == 2) else freqs_table(freqs)
    if ft.shape[0] < 1 or S % ft.shape[0] or ft.shape[1] * 2 != D:
        raise ValueError(f"freqs must be [S={S},1,{D // 2}] (or [F,1,{D // 2}] with F dividing S, "
                         f"row r using entry r % F), got {tuple(freqs.shape)}")
    ft = ft.to(q2.device).contiguous()
    if out is None:
        q_out = torch.empty(S, dim, dtype=torch.bfloat16, device=q2.device)
        k_out = torch.empty(S, dim, dtype=torch.bfloat16, device=q2.device)
    else:
        q_out, k_out = out
    cam = None
    cam_dim = 0
    if cam_tokens is not None:
        cam = _rows(cam_tokens).to(torch.bfloat16).contiguous()
        if cam.shape[0] != S:
            raise ValueError(
                f"camera tokens shape {tuple(cam_tokens.shape[:2])} must match q/k tokens {tuple(qx.shape[:2])}")
        cam_dim = cam.shape[1]
        cam_q_weight = cam_q_weight.to(torch.bfloat16).contiguous()
        cam_k_weight = cam_k_weight.to(torch.bfloat16).contiguous()
    nqw = norm_q_weight.to(torch.bfloat16).contiguous()
    nkw = norm_k_weight.to(torch.bfloat16).contiguous()
    for name, m in (("out_rows", out_rows), ("k_out_rows", k_out_rows)):
        if m is not None and (m.dtype != torch.int32 or m.numel() != S or m.device != q2.device):
            raise ValueError(f"{name} must be int32 [{S}] on {q2.device}")
    if q_out.stride(0) != k_out.stride(0):
        raise ValueError("q and k outputs must share a row stride")
    check(_lib.lib().hier_prep_qk(
        ptr(q2), ptr(k2), q2.stride(0), ptr(cam), cam_dim, ptr(cam_q_weight), ptr(cam_k_weight),
        ptr(nqw), ptr(nkw), ptr(ft), ft.shape[0], S, num_heads, D, float(eps), ptr(q_out), ptr(k_out),
        q_out.stride(0), ptr(out_rows), ptr(k_out_rows), stream_ptr(q2.device)))
    return q_out, k_out


class AttentionPlan:
    """Generic attention work plan: query pairs, key tiles, row bitmasks.

    ``q_pairs`` int32 ``[n,8]`` = (q_start0, q_rows0, q_start1, q_rows1,
    kv_begin, kv_end, 0, 0); ``kv_tiles`` int32 ``[m,4]`` = (k_row0, k_row1,
    mask0, mask1) with mask -1 full, -2 skip, else a row-mask index;
    ``row_masks`` int32 ``[k,128,4]``; ``order`` int32 ``[n]`` (or None)."""

    def __init__(self, q_pairs, kv_tiles, row_masks, order=None):
        self.q_pairs = q_pairs
        self.kv_tiles = kv_tiles
        self.row_masks = row_masks
        self.order = order


PLAN_CHECK_ENV = "MULTICS_B200_CHECK_PLANS"

_PLAN_CHECK_BITS = ((1, "a pair's key-tile range leaves the tile table"),
                    (2, "query rows leave the query tensor"),
                    (4, "a mask selector leaves the row-mask table"),
                    (8, "a key box starts outside its key/value stream"),
                    (16, "an order entry leaves the pairs"))


def check_plan(plan, q_rows: int, kv_rows, *, n_masks: Optional[int] = None,
               n_tiles: Optional[int] = None):
    """Raise ValueError when an attention plan's indices leave its tables or
    the tensors it will read (``hier_plan_check`` on the device, then one host
    read): the check to run before launching a plan that was built, stored or
    received elsewhere.  ``kv_rows``: rows of the key/value stream, or a list
    of them (one per stream)."""
    qp, kv = plan.q_pairs, plan.kv_tiles
    dev = qp.device
    rows = [int(kv_rows)] if isinstance(kv_rows, (int, np.integer)) else [int(r) for r in kv_rows]
    arr = (ctypes.c_int64 * len(rows))(*rows)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(_lib.lib().hier_plan_check(
        ptr(qp), qp.shape[0], ptr(kv), kv.shape[0] if n_tiles is None else int(n_tiles),
        plan.row_masks.shape[0] if n_masks is None else int(n_masks), ptr(plan.order),
        int(q_rows), arr, len(rows), ptr(status), stream_ptr(dev)))
    bits = int(status.item())
    if bits:
        raise ValueError("attention plan rejected before launch: " +
                         "; ".join(msg for bit, msg in _PLAN_CHECK_BITS if bits & bit))


def attention_from_plan(q, k, v, plan, num_heads, *, out=None, softmax_scale=None,
                        q_rows_total=None):
    """Run the tcgen05 attention kernel for ``plan`` on ``[S,H*D]`` bf16 rows.
    With ``MULTICS_B200_CHECK_PLANS=1`` the plan is bounds-checked first
    (:func:`check_plan`)."""
    q2, k2, v2 = _rows(q), _rows(k), _rows(v)
    for name, t in (("q", q2), ("k", k2), ("v", v2)):
        if t.dtype != torch.bfloat16:
            raise NotImplementedError(f"hierarchical B200 attention requires bf16 {name}; got {t.dtype}")
        if not t.is_cuda:
            raise NotImplementedError("hierarchical B200 attention requires CUDA tensors")
    if k2.stride(0) != v2.stride(0) or k2.shape != v2.shape:
        raise ValueError(f"K/V pools must match, got {tuple(k2.shape)} and {tuple(v2.shape)}")
    S, dim = q2.shape
    D = dim // num_heads
    if out is None:
        out = torch.empty(S, dim, dtype=torch.bfloat16, device=q2.device)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    n_pairs = plan.q_pairs.shape[0]
    if os.environ.get(PLAN_CHECK_ENV, "0") == "1":
        check_plan(plan, S if q_rows_total is None else q_rows_total, k2.shape[0])
    check(_lib.lib().hier_attn_fwd(
        ptr(q2), S if q_rows_total is None else q_rows_total, q2.stride(0), ptr(k2), ptr(v2),
        k2.shape[0], k2.stride(0), ptr(out), out.stride(0), num_heads, D, ptr(plan.q_pairs),
        n_pairs, ptr(plan.kv_tiles), ptr(plan.row_masks), ptr(plan.order), scale,
        ptr(_dev_err(q2.device)), stream_ptr(q2.device)))
    return out


class HierSequencePlan:
    """Full-sequence attention plan of one labels grouping on one GPU (the
    player-shard plan with a single shard, ``hier_shard_count`` / ``hier_shard_build``).

    Each player's rows run as 256-row strips (two 128-row query tiles) over
    exactly the key units their rows attend to (own history, group-mate
    frames of the blocks, the group's hub tokens); hub query rows run in
    128-row tiles of one group's frames.  Tiles that some rows see only in
    part carry per-row masks.  The plan's row order is the sequence order with the
    hub rows group-major (``ShardTopology.hub_rows_order``): the prologue
    writes q and k in that order (``seq_to_plan``), ``v``'s hub rows are
    gathered into it, and the kernel writes every player output row back to
    its sequence row (``plan_to_seq``).  Hub rows are computed as partial rows
    (per member player, and over the hub tokens) and merged into their
    sequence rows from their log-sum-exp.  Same edges as the block plan, so the same
    results up to the order of floating-point sums."""

    def __init__(self, spec, num_heads: int, page_table=None):
        from .sharded import ShardedHierAttention, ShardTopology

        if not HierSequencePlan.supports(spec):
            raise ValueError("HierSequencePlan needs a labels grouping without the no-local "
                             "topology, T % n_block == 0 and local_attn -1 or >= n_block")
        dev = spec.active.device
        topo = ShardTopology(P=spec.P, T=spec.T, L=spec.L, N=spec.N, KL=spec.KL, KG=spec.KG,
                             n_block=spec.n_block, local_attn=spec.local_attn,
                             direct=spec.direct, labels=spec.labels.cpu().numpy(), world=1,
                             rank=0)
        self.topo = topo
        self.num_heads = num_heads
        self.core = ShardedHierAttention(topo, num_heads, dev, active=spec.active,
                                         page_table=page_table)
        order = topo.local_rows()  # plan row -> sequence row
        inv = np.empty_like(order)
        inv[order] = np.arange(order.size)
        self.A = topo.own_rows
        self.S = int(order.size)
        self.plan_to_seq = torch.from_numpy(order.astype(np.int32)).to(dev)
        self.seq_to_plan = torch.from_numpy(inv.astype(np.int32)).to(dev)
        self.hub_src = torch.from_numpy((order[self.A:] - self.A).astype(np.int64)).to(dev)
        self.hub_dst = self.plan_to_seq[self.A:].contiguous()
        self.paged = page_table is not None
        if self.paged:
            # key/value pool: the player rows in 64-row pages, then the hub
            # rows in plan order; pool_rows[r] = pool row of sequence row r
            pt = torch.as_tensor(page_table).to(torch.int64).cpu()
            if pt.numel() * 64 < self.A:
                raise ValueError(f"page table of {pt.numel()} pages is short of {self.A} rows")
            base = self.core.page_rows
            plan = np.arange(self.S)
            phys = np.empty(self.S, np.int64)
            pr = plan[:self.A]
            phys[:self.A] = pt.numpy()[pr // 64] * 64 + pr % 64
            phys[self.A:] = base + (plan[self.A:] - self.A)
            self.pool_size = base + (self.S - self.A)
            self.pool_rows = torch.from_numpy(phys[inv].astype(np.int32)).to(dev)
        self.core.check_status()

    def to_pool(self, x):
        """A sequence-order ``[S, H*D]`` tensor laid out as this paged plan's
        key/value pool (the layout the prologue writes k into)."""
        pool = torch.zeros((self.pool_size, x.shape[1]), dtype=x.dtype, device=x.device)
        pool.index_copy_(0, self.pool_rows.long(), _rows(x))
        return pool

    def attend_paged(self, q_plan, k_pool, v_pool, out=None):
        """Attention of a paged plan: ``q_plan`` in plan row order, ``k_pool``
        / ``v_pool`` in the pool layout (:meth:`to_pool`); returns ``out`` in
        sequence order."""
        if not self.paged:
            raise ValueError("attend_paged needs a plan built with a page table")
        if out is None:
            out = torch.empty((self.S, q_plan.shape[1]), dtype=q_plan.dtype, device=q_plan.device)
        base = self.core.page_rows
        self.core.attend(q_plan, k_pool, v_pool, out, v_hub=v_pool[base:base + self.S - self.A],
                         out_rows=self.plan_to_seq)
        self.core.merge(out, out_rows=self.hub_dst)
        return out

    @staticmethod
    def supports(spec) -> bool:
        return (spec is not None and spec.membership is None and spec.labels is not None and not spec.no_local
                and spec.T % spec.n_block == 0
                and (spec.local_attn == -1 or spec.local_attn >= spec.n_block))

    def attend(self, q_plan, k_plan, v, out=None, events=None, lse=None):
        """Attention of roped ``q_plan`` / ``k_plan`` (plan row order) and
        ``v`` (sequence order), all ``[S, H*D]`` bf16; returns ``out`` in
        sequence order.  ``events`` (two CUDA events) are recorded on the
        current stream around the attention kernel's launch alone.  ``lse``
        (float32 ``[S, H]``, optional) receives every row's log2-sum-exp in
        sequence order (:meth:`hub_lse` for the hub rows)."""
        if out is None:
            out = torch.empty_like(v)
        v_hub = v[self.A:].index_select(0, self.hub_src)
        if events is not None:
            events[0].record()
        self.core.attend(q_plan, k_plan, v, out, v_hub=v_hub, out_rows=self.plan_to_seq, lse=lse)
        if events is not None:
            events[1].record()
        self.core.merge(out, out_rows=self.hub_dst)
        if lse is not None:
            self.hub_lse(lse)
        return out

    def hub_lse(self, lse):
        """The hub rows' log2-sum-exp over all their keys, log2 of the sum of
        2^lse over their partial rows (the merge's lists), into ``lse`` at
        their sequence rows."""
        c = self.core
        if not self.hub_dst.numel():
            return lse
        if getattr(self, "_lse_gather", None) is None:
            off = c.csr_off.long()
            counts = off[1:] - off[:-1]
            kmax = max(int(counts.max().item()), 1)
            idx = off[:-1, None] + torch.arange(kmax, device=off.device)[None]
            valid = idx < off[1:, None]
            rows = c.csr_rows.long()[torch.where(valid, idx, torch.zeros_like(idx))]
            self._lse_gather = (rows, valid)
        rows, valid = self._lse_gather
        vals = c.part_lse[rows]  # [hub rows, partials, H]
        vals = torch.where(valid[..., None], vals, torch.full_like(vals, float("-inf")))
        ln2 = math.log(2.0)
        lse[self.hub_dst.long()] = torch.logsumexp(vals * ln2, dim=1) / ln2
        return lse


def sequence_plan(block_mask: HierBlockMask, num_heads: int) -> Optional[HierSequencePlan]:
    """The :class:`HierSequencePlan` of ``block_mask``'s grouping (built once
    per mask and head count), or None when the grouping needs the block plan
    or ``MULTICS_B200_FULL_SEQUENCE_PLAN=blocks``."""
    mode = os.environ.get(FULL_SEQUENCE_PLAN_ENV, "segments")
    if mode not in ("segments", "blocks"):
        raise ValueError(f"{FULL_SEQUENCE_PLAN_ENV} must be 'segments' or 'blocks', got {mode!r}")
    if mode == "blocks" or not HierSequencePlan.supports(block_mask.spec):
        return None
    plans = block_mask.__dict__.setdefault("_sequence_plans", {})
    if num_heads not in plans:
        plans[num_heads] = HierSequencePlan(block_mask.spec, num_heads)
    return plans[num_heads]


def hier_block_attention(q, k, v, block_mask: HierBlockMask, num_heads, *, out=None):
    """Attention of roped ``q``/``k`` and ``v`` (``[1,S,H*D]`` or ``[S,H*D]``)
    under a :class:`HierBlockMask`; returns ``[1,S,H*D]`` bf16."""
    o = attention_from_plan(q, k, v, block_mask, num_heads, out=out)
    return o.unsqueeze(0)


def hier_attention_layer(qx, kx, v, freqs, block_mask: HierBlockMask, num_heads, *,
                         norm_q_weight, norm_k_weight, cam_tokens=None, cam_q_weight=None,
                         cam_k_weight=None, eps=1e-6, out=None):
    """One hierarchical attention layer after the q/k/v projections: fused
    camera + RMSNorm + RoPE prologue, then block-sparse attention.  Equivalent
    to the reference's ``_project_self_attn_qkv`` tail + ``flash_attention(mask)``
    (``attention.py:355-365,39-54``); returns ``[S, H*D]`` bf16."""
    block_mask = attention_mask_plan(block_mask, _rows(qx).shape[0], qx.device)
    sp = sequence_plan(block_mask, num_heads)
    q, k = hier_prep_qk(qx, kx, freqs, num_heads, norm_q_weight=norm_q_weight,
                        norm_k_weight=norm_k_weight, cam_tokens=cam_tokens,
                        cam_q_weight=cam_q_weight, cam_k_weight=cam_k_weight, eps=eps,
                        out_rows=None if sp is None else sp.seq_to_plan)
    if sp is not None:
        return sp.attend(q, k, _rows(v), out)
    return attention_from_plan(q, k, v, block_mask, num_heads, out=out)


_DENSE_PLANS: list = []  # [(weakref to mask or None, version, S, device, HierBlockMask)]


def attention_mask_plan(mask, S: int, device) -> HierBlockMask:
    """The block mask / work plan for ``mask`` as :meth:`SelfAttention.forward`
    accepts it.  Plans of dense masks are kept for the two most recent masks
    (and for no mask per length), like the reference's bounded mask caches,
    and rebuilt when the mask tensor is modified in place."""
    import weakref

    if isinstance(mask, HierBlockMask):
        return mask
    spec = getattr(mask, "hier_spec", None)
    if spec is not None:
        return block_mask_for_spec(spec)
    if mask is not None and not isinstance(mask, torch.Tensor):
        raise TypeError(f"mask must be a HierBlockMask, a dense [S,S] tensor or None; got "
                        f"{type(mask).__name__}")
    dev = torch.device(device)
    for ref, ver, s_, d_, bm in _DENSE_PLANS:
        if s_ != S or d_ != dev:
            continue
        if mask is None and ref is None:
            return bm
        if mask is not None and ref is not None and ref() is mask and mask._version == ver:
            return bm
    bm = build_dense_block_plan(mask, S, dev)
    _DENSE_PLANS.insert(0, (None if mask is None else weakref.ref(mask),
                            None if mask is None else mask._version, S, dev, bm))
    del _DENSE_PLANS[2:]
    return bm


def _rope_torch(x, freqs, num_heads):
    """``rope_apply`` (``rope.py:248-254``) as differentiable PyTorch
    operations: complex multiply in float64, cast back.  ``freqs`` complex
    ``[S, 1, D/2]`` or a float ``[S, D/2, 2]`` (cos, sin) table."""
    if not torch.is_complex(freqs):
        f = freqs.reshape(freqs.shape[0], -1, 2).double()
        freqs = torch.complex(f[..., 0], f[..., 1])
    b, s, nd = x.shape
    xc = torch.view_as_complex(x.double().reshape(b, s, num_heads, nd // num_heads // 2, 2))
    out = torch.view_as_real(xc * freqs.reshape(s, 1, -1).to(xc.device)).flatten(3)
    return out.reshape(b, s, nd).to(x.dtype)


class RMSNorm(nn.Module):
    """``attention.py:231-242``: fp32 ``x*rsqrt(mean(x^2)+eps)`` then ``*weight``."""

    def __init__(self, dim, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        dtype = x.dtype
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)).to(dtype) * self.weight


class SelfAttention(nn.Module):
    """Hierarchical self-attention module with the reference's constructor and
    ``forward(x, freqs, mask=None, cam_tokens=None)`` signature
    (``attention.py:255-442``).

    ``mask`` is a :class:`HierBlockMask`
    (``multics_b200.hier_masks.build_stage2_hier_flex_block_mask``), a dense
    bool mask (``build_stage2_hier_self_attn_mask`` or any other) or None, as
    the reference's Flex and sdpa call sites pass.  The q/k/v/o
    projections run as cuBLAS GEMMs; the camera add, both RMSNorms and RoPE
    run in one prologue kernel and the attention in the tcgen05 kernel."""

    def __init__(self, dim: int, num_heads: int, eps: float = 1e-6):
        super().__init__()
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        self.norm_q = RMSNorm(dim, eps=eps)
        self.norm_k = RMSNorm(dim, eps=eps)
        self.sink_size = 0
        self.local_attn_size = 6
        self.num_frame_per_block = 7
        self.attn_impl = "b200"
        self.cam_dim = None
        self.cam_q = None
        self.cam_k = None
        self.cam_dropout_p = 0.0

    def enable_camera_pose_qk(self, cam_dim: int, dropout_p: float = 0.1):
        """Zero-initialised, bias-free camera adapters on Q/K (``attention.py:278-305``)."""
        cam_dim = int(cam_dim)
        dropout_p = float(dropout_p)
        if not 0.0 <= dropout_p < 1.0:
            raise ValueError(f"camera dropout_p must be in [0,1), got {dropout_p}")
        if self.cam_q is not None and self.cam_dim == cam_dim:
            self.cam_dropout_p = dropout_p
            return
        dev, dt = self.q.weight.device, self.q.weight.dtype
        self.cam_dim = cam_dim
        self.cam_dropout_p = dropout_p
        self.cam_q = nn.Linear(cam_dim, self.dim, bias=False).to(device=dev, dtype=dt)
        self.cam_k = nn.Linear(cam_dim, self.dim, bias=False).to(device=dev, dtype=dt)
        nn.init.zeros_(self.cam_q.weight)
        nn.init.zeros_(self.cam_k.weight)

    def project_qkv(self, x, freqs, cam_tokens=None, out_rows=None):
        """Projected + fused-prologue ``(q, k, v)`` as ``[S, dim]`` bf16 rows
        (``out_rows``: the row of each token in q and k, see :func:`hier_prep_qk`)."""
        if cam_tokens is not None and (self.cam_q is None or self.cam_k is None):
            raise RuntimeError("camera_pose was provided but enable_camera_pose_qk() was not called")
        if cam_tokens is not None and cam_tokens.shape[:2] != x.shape[:2]:
            raise ValueError(
                f"camera tokens shape {tuple(cam_tokens.shape[:2])} must match q/k tokens {tuple(x.shape[:2])}")
        if cam_tokens is not None and self.training and self.cam_dropout_p > 0:
            cam_tokens = torch.nn.functional.dropout(cam_tokens, p=self.cam_dropout_p, training=True)
        qx = self.q(x)
        kx = self.k(x)
        v = self.v(x)
        q, k = hier_prep_qk(
            qx, kx, freqs, self.num_heads, norm_q_weight=self.norm_q.weight,
            norm_k_weight=self.norm_k.weight, cam_tokens=cam_tokens,
            cam_q_weight=None if self.cam_q is None else self.cam_q.weight,
            cam_k_weight=None if self.cam_k is None else self.cam_k.weight, eps=self.norm_q.eps,
            out_rows=out_rows)
        return q, k, _rows(v)

    def forward(self, x, freqs, mask=None, cam_tokens=None):
        """``attention.py:436-442``.  ``mask`` is what the reference's call
        sites pass: the :class:`HierBlockMask` of
        ``build_stage2_hier_flex_block_mask`` (the Flex path), the dense bool
        mask of ``build_stage2_hier_self_attn_mask`` (the sdpa path; it
        carries its grouping and runs on the grouping's plan), any other dense
        ``[S,S]`` mask (block plan built from its bytes), or None (unmasked).
        A batch ``x`` ``[B, L, dim]`` with ``B > 1`` is the DiT block's
        per-frame action attention (``blocks.py:684-686``): ``mask`` is one
        ``[L, L]`` mask shared by the batch and ``freqs`` ``[L, 1, D/2]``.
        While autograd records (training), the call runs
        :meth:`_forward_train` (or :meth:`_forward_batch` with the fused
        prologue's backward): the attention on an aligned plan with its B200
        backward."""
        train = torch.is_grad_enabled() and (x.requires_grad or any(
            p.requires_grad for p in self.parameters()))
        if x.dim() == 3 and x.shape[0] > 1:
            return self._forward_batch(x, freqs, mask, cam_tokens, train=train)
        if train:
            return self._forward_train(x, freqs, mask, cam_tokens)
        mask = attention_mask_plan(mask, x.shape[1], x.device)
        sp = sequence_plan(mask, self.num_heads)
        q, k, v = self.project_qkv(x, freqs, cam_tokens,
                                   out_rows=None if sp is None else sp.seq_to_plan)
        if sp is not None:
            out = sp.attend(q, k, v)
        else:
            out = attention_from_plan(q, k, v, mask, self.num_heads)
        return self.o(out.unsqueeze(0))


    def _forward_train(self, x, freqs, mask, cam_tokens):
        """Differentiable forward (``attention.py:355-365,436-442`` with
        autograd): the projections (cuBLAS), the camera add + RMSNorm + RoPE
        prologue and its backward as fused kernels
        (:func:`multics_b200.train.prologue_grad`), the attention on the block
        plan through :func:`multics_b200.train.hier_block_attention_grad`
        (tcgen05 forward and backward kernels)."""
        from .train import hier_block_attention_grad, prologue_grad

        if cam_tokens is not None and (self.cam_q is None or self.cam_k is None):
            raise RuntimeError("camera_pose was provided but enable_camera_pose_qk() was not called")
        if cam_tokens is not None and cam_tokens.shape[:2] != x.shape[:2]:
            raise ValueError(f"camera tokens shape {tuple(cam_tokens.shape[:2])} must match "
                             f"q/k tokens {tuple(x.shape[:2])}")
        if cam_tokens is not None and self.training and self.cam_dropout_p > 0:
            cam_tokens = torch.nn.functional.dropout(cam_tokens, p=self.cam_dropout_p, training=True)
        qx, kx, v = self.q(x), self.k(x), self.v(x)
        q, k = prologue_grad(qx, kx, freqs, self.num_heads, norm_q_weight=self.norm_q.weight,
                             norm_k_weight=self.norm_k.weight, cam_tokens=cam_tokens,
                             cam_q_weight=None if self.cam_q is None else self.cam_q.weight,
                             cam_k_weight=None if self.cam_k is None else self.cam_k.weight,
                             eps=self.norm_q.eps)
        bm = attention_mask_plan(mask, x.shape[1], x.device)
        out = hier_block_attention_grad(q, k, _rows(v), bm, self.num_heads)
        return self.o(out.view(x.shape))

    def _forward_batch(self, x, freqs, mask, cam_tokens, train=False):
        """``B`` sequences of ``L`` tokens under one shared mask: projections,
        the fused prologue over the ``B*L`` rows (RoPE table row ``r % L``)
        and the shared-mask attention plan.  ``train``: the prologue and the
        attention with their backward kernels (:func:`multics_b200.train.prologue_grad`,
        the aligned shared-mask plan)."""
        from .action import shared_mask_attention

        B, L, dim = x.shape
        if cam_tokens is not None:
            if self.cam_q is None or self.cam_k is None:
                raise RuntimeError("camera_pose was provided but enable_camera_pose_qk() was not called")
            if cam_tokens.shape[:2] != x.shape[:2]:
                raise ValueError(f"camera tokens shape {tuple(cam_tokens.shape[:2])} must match "
                                 f"q/k tokens {tuple(x.shape[:2])}")
            cam_tokens = cam_tokens.reshape(B * L, -1)
            if self.training and self.cam_dropout_p > 0:
                cam_tokens = torch.nn.functional.dropout(cam_tokens, p=self.cam_dropout_p,
                                                         training=True)
        if train:
            from .train import prologue_grad
            prep = prologue_grad
        else:
            prep = hier_prep_qk
        q, k = prep(
            self.q(x).reshape(B * L, dim), self.k(x).reshape(B * L, dim), freqs, self.num_heads,
            norm_q_weight=self.norm_q.weight, norm_k_weight=self.norm_k.weight,
            cam_tokens=cam_tokens, cam_q_weight=None if self.cam_q is None else self.cam_q.weight,
            cam_k_weight=None if self.cam_k is None else self.cam_k.weight, eps=self.norm_q.eps)
        out = shared_mask_attention(q.view(B, L, dim), k.view(B, L, dim), self.v(x),
                                    self.num_heads, mask)
        return self.o(out)


class CrossAttention(nn.Module):
    """The reference's ``CrossAttention`` (``attention.py:1046-1090``): same
    constructor, parameters and ``forward(x, y, mask=None)``.  q from ``x``,
    k and v from the context ``y`` (after 257 image tokens when
    ``has_image_input``), RMSNorm on q and k, no RoPE; the attention runs on
    the tcgen05 kernel with ``mask`` shared by the batch (the keyboard
    cross-attention's repeated frame mask, ``blocks.py:692-697``) or
    unmasked (the text cross-attention)."""

    def __init__(self, dim: int, num_heads: int, eps: float = 1e-6,
                 has_image_input: bool = False):
        super().__init__()
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.q = nn.Linear(dim, dim)
        self.k = nn.Linear(dim, dim)
        self.v = nn.Linear(dim, dim)
        self.o = nn.Linear(dim, dim)
        self.norm_q = RMSNorm(dim, eps=eps)
        self.norm_k = RMSNorm(dim, eps=eps)
        self.has_image_input = has_image_input
        if has_image_input:
            self.k_img = nn.Linear(dim, dim)
            self.v_img = nn.Linear(dim, dim)
            self.norm_k_img = RMSNorm(dim, eps=eps)

    def forward(self, x, y, mask=None):
        from .action import shared_mask_attention

        if self.has_image_input:
            img, ctx = y[:, :257], y[:, 257:]
        else:
            ctx = y
        q = self.norm_q(self.q(x))
        k = self.norm_k(self.k(ctx))
        v = self.v(ctx)
        out = shared_mask_attention(q, k, v, self.num_heads, mask)
        if self.has_image_input:
            k_img = self.norm_k_img(self.k_img(img))
            v_img = self.v_img(img)
            out = out + shared_mask_attention(q, k_img, v_img, self.num_heads, mask)
        return self.o(out)


_INFER_KERNELS = ("sdpa", "segmented", "tiled128", "packed_varlen", "paged_kv")


def _causal_forward_hier_hub(self, x, freqs, kv_cache, current_start=0, num_frames=None,
                             num_players=None, num_hub_tokens=None, cam_tokens=None,
                             group_labels=None, active_group=None, direct_player=False,
                             membership=None, global_only=None):
    """Cached hierarchical self-attention of one block of ``num_frames`` new
    frames (``SelfAttention.causal_forward_hier_hub``,
    ``multics/models/attention.py:456-1005``): projections, the fused
    camera/RMSNorm/RoPE prologue, rolling-cache appends in the reference's
    cache format, then the tcgen05 attention over the caches in place and the
    output projection.  Every ``WAN_HIER_INFER_KERNEL`` value selects the same
    B200 kernel; the reference's value checks and refusals are kept."""
    import os

    from .cached import hierarchical_cached_attention
    from .hier_masks import (_prepare_hier_group_tensors, _prepare_hier_membership_tensors,
                             _refuse_membership_on_scalar_kernel)
    from .kv_cache import rolling_bool_cache_append, rolling_cache_append

    b, s = x.shape[:2]
    H, D = self.num_heads, self.head_dim
    P = int(num_players if num_players is not None else kv_cache["num_players"])
    N = int(kv_cache["num_groups"])
    KL = int(kv_cache["num_local_hub_tokens"])
    KG = int(kv_cache["num_global_hub_tokens"])
    no_local = bool(getattr(self, "hier_no_local_hub", False))
    if bool(kv_cache.get("hier_no_local_hub", False)) != no_local:
        raise ValueError("hier_no_local_hub mismatch between SelfAttention and KV cache")
    n_frames = int(num_frames)
    K_total = int(num_hub_tokens if num_hub_tokens is not None else N * KL + KG)
    if K_total != N * KL + KG:
        raise ValueError(f"hier_hub K_total mismatch: {K_total} != {N}*{KL}+{KG}")
    if no_local and (KL != 0 or KG <= 0):
        raise ValueError(
            f"hier_no_local_hub cached attention requires K_L=0 and K_G>0; got K_L={KL}, K_G={KG}")
    use_membership = membership is not None
    mem_full = go_full = None
    if use_membership:
        mem_full, go_full, active = _prepare_hier_membership_tensors(
            membership, global_only, active_group, P, n_frames, N, x.device, allow_full_t=True)
        labels = None
    else:
        labels, active = _prepare_hier_group_tensors(group_labels, active_group, P, n_frames, N,
                                                     x.device)
        if n_frames > 1 and labels.numel() and not torch.equal(labels,
                                                               labels[:1].expand_as(labels)):
            raise ValueError(
                "hier_hub cached inference requires group_labels constant inside each latent block")
    hub_len = n_frames * K_total
    agent_len = s - hub_len
    if agent_len <= 0 or agent_len % (P * n_frames) != 0:
        raise ValueError(
            f"hier_hub causal seq shape invalid: S={s}, hub_len={hub_len}, P={P}, n={n_frames}")
    L = agent_len // (P * n_frames)
    n_block = int(self.num_frame_per_block)
    local_attn = int(self.local_attn_size)
    dev = x.device
    if freqs.shape[0] != s:
        raise ValueError("hier_hub causal_forward expects freqs.shape[0] == seq_len")
    if b != 1:
        raise NotImplementedError(f"B200 cached hierarchical inference supports B=1; got B={b}")
    kernel = os.environ.get("WAN_HIER_INFER_KERNEL", "sdpa").strip().lower()
    if kernel not in _INFER_KERNELS:
        raise ValueError(
            "WAN_HIER_INFER_KERNEL must be 'sdpa', 'segmented', 'tiled128', 'packed_varlen', "
            f"or 'paged_kv', got {kernel!r}")
    if kernel in ("segmented", "tiled128"):
        if no_local:
            raise NotImplementedError(
                "hier_no_local_hub cached inference supports sdpa, packed_varlen, or paged_kv; got "
                + kernel)
        if use_membership:
            _refuse_membership_on_scalar_kernel(infer_kernel=kernel)

    q, k, v = self.project_qkv(x, freqs, cam_tokens)  # [s, H*D] rows, roped q/k
    q4, k4, v4 = (t.view(1, s, H, D) for t in (q, k, v))
    local_start = agent_len
    global_start = agent_len + n_frames * N * KL
    retention = local_attn + n_frames if local_attn != -1 else -1
    start_frame = current_start // max(P * L, 1)
    end_frame = start_frame + n_frames - 1
    if use_membership:
        T_full = int(mem_full.shape[0])
        if start_frame < 0 or start_frame + n_frames > T_full:
            raise ValueError(f"hier_hub membership T={T_full} does not cover cached block "
                             f"[{start_frame},{start_frame + n_frames})")
        mem_blk = mem_full[start_frame:start_frame + n_frames]
        go_blk = go_full[start_frame:start_frame + n_frames]
        active = active[start_frame:start_frame + n_frames]
        if n_frames > 1:
            if not torch.equal(mem_blk, mem_blk[:1].expand_as(mem_blk)):
                raise ValueError(
                    "hier_hub cached inference requires membership constant inside each latent block")
            if not torch.equal(go_blk, go_blk[:1].expand_as(go_blk)):
                raise ValueError(
                    "hier_hub cached inference requires global_only constant inside each latent block")
    # append this block's keys/values to the rolling caches
    agent_k = k4[:, :agent_len].reshape(1, P, n_frames * L, H, D)
    agent_v = v4[:, :agent_len].reshape(1, P, n_frames * L, H, D)
    for p in range(P):
        rolling_cache_append(kv_cache["agent_caches"][p], agent_k[:, p], agent_v[:, p],
                             start_frame * L, (start_frame + n_frames) * L, retention, 0, L)
    if not no_local:
        loc_k = k4[:, local_start:global_start].reshape(1, n_frames, N, KL, H, D)
        loc_v = v4[:, local_start:global_start].reshape(1, n_frames, N, KL, H, D)
        for g in range(N):
            c = kv_cache["local_hubs"][g]
            rolling_bool_cache_append(c, "active", active[:, g].repeat_interleave(KL),
                                      start_frame * KL, (start_frame + n_frames) * KL,
                                      retention, 0, KL)
            rolling_cache_append(c, loc_k[:, :, g].reshape(1, n_frames * KL, H, D),
                                 loc_v[:, :, g].reshape(1, n_frames * KL, H, D),
                                 start_frame * KL, (start_frame + n_frames) * KL, retention, 0, KL)
    if KG > 0:
        rolling_cache_append(kv_cache["global_hub"], k4[:, global_start:], v4[:, global_start:],
                             start_frame * KG, (start_frame + n_frames) * KG, retention, 0, KG)

    def window(cache, tpf):
        end = int(cache["local_end_index"].item())
        held = end // tpf if tpf > 0 else 0
        frames = (end_frame - held + 1) + torch.arange(end, device=dev) // max(tpf, 1)
        return frames, cache["k"][:, :end].reshape(1, end, H * D), \
            cache["v"][:, :end].reshape(1, end, H * D)

    agent = [window(c, L) for c in kv_cache["agent_caches"]]
    local, local_active = [], []
    if not no_local:
        for c in kv_cache["local_hubs"]:
            f, kk, vv = window(c, KL)
            local.append((f, kk, vv))
            act = c.get("active")
            local_active.append(torch.ones(f.shape[0], device=dev, dtype=torch.bool) if act is None
                                else act[:f.shape[0]].to(device=dev, dtype=torch.bool))
    if KG > 0:
        gf, gk, gv = window(kv_cache["global_hub"], KG)
    else:
        gf = torch.empty(0, device=dev, dtype=torch.long)
        gk = gv = x.new_zeros(1, 0, H * D)
    out = hierarchical_cached_attention(
        roped_q=q4, agent_frames=[a[0] for a in agent], agent_keys=[a[1] for a in agent],
        agent_vals=[a[2] for a in agent], local_frames=[t[0] for t in local],
        local_keys=[t[1] for t in local], local_vals=[t[2] for t in local],
        local_active_tokens=local_active, global_frames=gf, global_keys=gk, global_vals=gv,
        labels=labels, active=active, P=P, N=N, L=L, KL=KL, KG=KG, n_frames=n_frames,
        n_block=n_block, local_attn=local_attn, direct_player=direct_player,
        membership=mem_full if use_membership else None,
        global_only=go_full if use_membership else None, hier_no_local_hub=no_local)
    return self.o(out.type_as(self.o.weight))


SelfAttention.causal_forward_hier_hub = _causal_forward_hier_hub

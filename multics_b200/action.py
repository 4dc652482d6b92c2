"""Action-branch attention of the Multics DiT block on B200.

After its hierarchical self-attention, the reference's DiT block
(``multics/models/blocks.py:587-700``) runs two more masked attentions, both
through ``flash_attention(q, k, v, num_heads, mask)`` (``attention.py:39-54``)
with one small bool mask broadcast over a batch:

* the per-frame mouse ("temporal") attention ``action_temporal_attn``, a copy
  of ``SelfAttention`` applied to ``[players * patches, frames, dim]`` with a
  1-D RoPE over frames and the mask ``get_temporal_block_causal_mask``
  ``[frames, frames]`` (``hier_masks.py:1152-1166``; ``blocks.py:441-447,
  677-691``);
* the keyboard cross-attention ``action_cross_attn``, a ``CrossAttention``
  from ``[players, frames * patches, dim]`` to the keyboard tokens
  ``[players, frames * 12, dim]`` under the frame mask repeated to
  ``[frames * patches, frames * 12]`` (``blocks.py:446-448,692-697``);

and their KV-cached forms over a rolling window, whose masks compare the
current block's frames with the window's (``blocks.py:256-375``).

:func:`shared_mask_attention` is that call for any mask shared by the batch.
Its plan (:class:`SharedMaskPlan`, built on the GPU) packs short sequences
several to a 128-row tile with block-diagonal row masks, and it runs on the
same tcgen05 attention kernel as the hierarchical layer.
"""

from __future__ import annotations

import ctypes
import weakref
from typing import Optional

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr
from .attention import AttentionPlan, attention_from_plan

__all__ = ["get_temporal_block_causal_mask", "keyboard_frame_mask", "cached_frame_mask",
           "SharedMaskPlan", "shared_mask_plan", "shared_mask_attention"]


def get_temporal_block_causal_mask(num_frames: int, num_frame_per_block: int,
                                   local_attn_size: int, device=None) -> torch.Tensor:
    """Frame ``i`` sees frame ``j`` iff ``j``'s block is not after ``i``'s and
    ``i - j < local_attn_size`` (no window for -1); ``[F, F]`` bool
    (``hier_masks.py:1152-1166``)."""
    t = torch.arange(num_frames, device=device)
    m = (t[None, :] // num_frame_per_block) <= (t[:, None] // num_frame_per_block)
    if local_attn_size != -1:
        m = m & (t[:, None] - t[None, :] < local_attn_size)
    return m


def keyboard_frame_mask(frame_mask: torch.Tensor, num_patches: int,
                        tokens_per_kbd_frame: int = 12) -> torch.Tensor:
    """The keyboard cross-attention mask: every frame's ``num_patches`` query
    rows see the ``tokens_per_kbd_frame`` keyboard tokens of every frame the
    frame mask allows, ``[F * num_patches, G * tokens_per_kbd_frame]``
    (``repeat(frame_mask, "f g -> (f q) (g k)")``, ``blocks.py:446-448``)."""
    return frame_mask.repeat_interleave(num_patches, 0).repeat_interleave(tokens_per_kbd_frame, 1)


def cached_frame_mask(query_frames: torch.Tensor, key_frames: torch.Tensor,
                      num_frame_per_block: int, local_attn_size: int) -> torch.Tensor:
    """Mask of the cached action attentions: global query frame ``gq`` sees
    global key frame ``gk`` iff ``gk // n <= gq // n`` and, with a window,
    ``gq - gk < local_attn_size`` (``blocks.py:300-305,366-371``)."""
    gq = query_frames.reshape(-1, 1)
    gk = key_frames.reshape(1, -1)
    m = gk // num_frame_per_block <= gq // num_frame_per_block
    if local_attn_size != -1:
        m = m & (gq - gk < local_attn_size)
    return m


class SharedMaskPlan(AttentionPlan):
    """Work plan of ``B`` independent attentions under one ``[Lq, Lk]`` mask:
    query row ``b*Lq + i`` sees key row ``b*Lk + j`` iff ``mask[i, j]``.
    Built on the GPU by ``hier_shared_mask_plan_build``; the fields are those
    of :class:`~multics_b200.attention.AttentionPlan` (per-row masks).
    ``aligned`` cuts the tiles on the 128-row grid of the flat rows, the form
    the backward kernels take (:func:`multics_b200.train.plan_attention_grad`)."""

    def __init__(self, mask: torch.Tensor, B: int, aligned: bool = False):
        if mask.dim() != 2:
            raise ValueError(f"shared mask must be [Lq, Lk], got {tuple(mask.shape)}")
        dev = mask.device
        if dev.type != "cuda":
            raise NotImplementedError("the shared-mask plan is built on a CUDA device")
        m = mask.to(torch.bool).contiguous().view(torch.uint8)
        Lq, Lk = m.shape
        lib = _lib.lib()
        n_pairs, cap = ctypes.c_int32(), ctypes.c_int32()
        check(lib.hier_shared_mask_plan_size(B, Lq, Lk, int(aligned), ctypes.byref(n_pairs),
                                             ctypes.byref(cap)))
        self.B, self.Lq, self.Lk, self.aligned = int(B), int(Lq), int(Lk), bool(aligned)
        self.n_pairs, self.tiles_per_pair = int(n_pairs.value), int(cap.value)
        n_ent = self.n_pairs * self.tiles_per_pair
        q_pairs = torch.empty((self.n_pairs, 8), dtype=torch.int32, device=dev)
        kv_tiles = torch.empty((n_ent, 4), dtype=torch.int32, device=dev)
        row_masks = torch.empty((2 * n_ent, 128, 4), dtype=torch.int32, device=dev)
        # the longest-first order is a quadratic ranking; beyond a few thousand
        # pairs (all of similar length here) the identity order is kept
        order = (torch.empty(self.n_pairs, dtype=torch.int32, device=dev)
                 if self.n_pairs <= 4096 else None)
        check(lib.hier_shared_mask_plan_build(
            ptr(m), m.stride(0), B, Lq, Lk, int(aligned), ptr(q_pairs), ptr(kv_tiles),
            ptr(row_masks), ptr(order), stream_ptr(dev)))
        super().__init__(q_pairs, kv_tiles, row_masks, order)
        self._mask_bytes = m  # read by the builder on the stream
        self._aligned_form = None

    def aligned_form(self) -> "SharedMaskPlan":
        """This plan's mask and batch as an aligned plan (itself when it is
        one), built once."""
        if self.aligned:
            return self
        if self._aligned_form is None:
            self._aligned_form = SharedMaskPlan(self._mask_bytes.view(torch.bool), self.B,
                                                aligned=True)
        return self._aligned_form


# (weakref to the caller's mask or None, its _version, B, Lq, Lk, device,
# aligned, plan): the most recent plans, as the reference's bounded mask caches
_PLANS = []
_PLAN_LIMIT = 8


def _shared_mask(mask, Lq: int, Lk: int, device) -> Optional[torch.Tensor]:
    """The caller's mask as ``[Lq, Lk]`` bool on ``device`` (leading size-1
    dimensions dropped, SDPA's broadcast applied), or None for no mask."""
    if mask is None:
        return None
    if not isinstance(mask, torch.Tensor):
        raise TypeError(f"mask must be a tensor or None, got {type(mask).__name__}")
    m = mask
    while m.dim() > 2:
        if m.shape[0] != 1:
            raise ValueError(
                f"mask {tuple(mask.shape)} varies over the batch or heads; this attention "
                f"takes one [Lq, Lk] mask shared by the batch")
        m = m[0]
    if m.dim() < 2:
        m = m.reshape(1, -1)
    try:
        m = m.expand(Lq, Lk)
    except RuntimeError:
        raise ValueError(f"mask {tuple(mask.shape)} does not broadcast to [{Lq}, {Lk}]") from None
    return m.to(device=device, dtype=torch.bool)


def shared_mask_plan(mask, B: int, Lq: int, Lk: int, device,
                     aligned: bool = False) -> SharedMaskPlan:
    """The plan for ``mask`` (any form :func:`shared_mask_attention` takes),
    reused while the same mask tensor is passed unmodified."""
    dev = torch.device(device)
    for ref, ver, b_, q_, k_, d_, a_, plan in _PLANS:
        if (b_, q_, k_, d_, a_) != (B, Lq, Lk, dev, bool(aligned)):
            continue
        if mask is None and ref is None:
            return plan
        if mask is not None and ref is not None and ref() is mask and mask._version == ver:
            return plan
    m = _shared_mask(mask, Lq, Lk, dev)
    if m is None:
        m = torch.ones((Lq, Lk), dtype=torch.bool, device=dev)
    plan = SharedMaskPlan(m, B, aligned)
    _PLANS.insert(0, (None if mask is None else weakref.ref(mask),
                      None if mask is None else mask._version, B, Lq, Lk, dev, bool(aligned),
                      plan))
    del _PLANS[_PLAN_LIMIT:]
    return plan


def shared_mask_attention(q, k, v, num_heads: int, mask=None, *, out=None,
                          plan: Optional[SharedMaskPlan] = None) -> torch.Tensor:
    """``flash_attention(q, k, v, num_heads, mask)`` (``attention.py:39-54``)
    for a mask shared by the batch, on the tcgen05 kernel.

    ``q`` bf16 ``[B, Lq, H*128]``, ``k``/``v`` bf16 ``[B, Lk, H*128]``;
    ``mask`` bool (or any dtype, read as ``mask.to(bool)``) ``[Lq, Lk]``, with
    optional leading size-1 dimensions or SDPA broadcasting, or None.
    Returns ``[B, Lq, H*128]`` bf16.  A query row that sees no key is 0 (SDPA
    gives NaN there).  While autograd records and ``q``, ``k`` or ``v``
    requires grad, the call is differentiable: the attention runs on the
    aligned form of the plan with the B200 backward kernels
    (:func:`multics_b200.train.plan_attention_grad`)."""
    if q.dim() != 3 or k.dim() != 3 or v.shape != k.shape:
        raise ValueError(f"expected q [B,Lq,dim] and k, v [B,Lk,dim]; got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    B, Lq, dim = q.shape
    Lk = k.shape[1]
    if k.shape[0] != B or k.shape[2] != dim:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} disagree")
    if dim % num_heads or dim // num_heads != 128:
        raise NotImplementedError(
            f"the B200 attention kernel needs head_dim 128; got dim {dim} over {num_heads} heads")
    grad = torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad)
    if plan is not None and (plan.B, plan.Lq, plan.Lk) != (B, Lq, Lk):
        raise ValueError(f"plan is for B={plan.B}, Lq={plan.Lq}, Lk={plan.Lk}")
    if grad:
        from .train import plan_attention_grad

        if out is not None:
            raise ValueError("out= is not supported while autograd records")
        # a caller's plan carries its own mask: its aligned form, not `mask`
        plan = (shared_mask_plan(mask, B, Lq, Lk, q.device, aligned=True) if plan is None
                else plan.aligned_form())
        res = plan_attention_grad(q.reshape(B * Lq, dim), k.reshape(B * Lk, dim),
                                  v.reshape(B * Lk, dim), plan, num_heads)
        return res.view(B, Lq, dim)
    if plan is None:
        plan = shared_mask_plan(mask, B, Lq, Lk, q.device)
    o = None if out is None else out.view(B * Lq, dim)
    res = attention_from_plan(q.reshape(B * Lq, dim), k.reshape(B * Lk, dim),
                              v.reshape(B * Lk, dim), plan, num_heads, out=o)
    return res.view(B, Lq, dim)

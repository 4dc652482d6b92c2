"""Hierarchical self-attention on B200: fused prologue + tcgen05 attention.

Drop-in counterparts of the reference's ``multics/models/attention.py``:

* :func:`hier_prep_qk` - camera Q/K add + RMSNorm + RoPE
  (``attention.py:307-365``, ``rope.py:248-254``) in one CUDA kernel;
* :func:`hier_block_attention` - attention over a :class:`HierBlockMask`
  (the role of ``flash_attention(mask)`` / FlexAttention,
  ``attention.py:39-54,322-353``);
* :class:`SelfAttention` - same constructor and ``forward(x, freqs, mask,
  cam_tokens)`` signature as the reference module (``attention.py:255-442``).
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from . import _lib
from ._lib import check, ptr, stream_ptr
from .hier_masks import HierBlockMask

__all__ = ["hier_prep_qk", "hier_block_attention", "freqs_table", "RMSNorm", "SelfAttention",
           "AttentionPlan", "attention_from_plan"]

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
                 cam_q_weight=None, cam_k_weight=None, eps=1e-6, out=None):
    """``q = rope(rmsnorm(qx + cam @ Wq^T) * wq)`` and the same for k, bf16.

    ``freqs``: complex ``[S,1,D/2]`` (as built by the reference's freq
    builders) or a float32 ``[S,D/2,2]`` table from :func:`freqs_table`."""
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
    if ft.shape[0] != S or ft.shape[1] * 2 != D:
        raise ValueError(f"freqs must be [S={S},1,{D // 2}], got {tuple(freqs.shape)}")
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
    check(_lib.lib().hier_prep_qk(
        ptr(q2), ptr(k2), q2.stride(0), ptr(cam), cam_dim, ptr(cam_q_weight), ptr(cam_k_weight),
        ptr(nqw), ptr(nkw), ptr(ft), S, num_heads, D, float(eps), ptr(q_out), ptr(k_out),
        q_out.stride(0), stream_ptr(q2.device)))
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


def attention_from_plan(q, k, v, plan, num_heads, *, out=None, softmax_scale=None,
                        q_rows_total=None):
    """Run the tcgen05 attention kernel for ``plan`` on ``[S,H*D]`` bf16 rows."""
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
    check(_lib.lib().hier_attn_fwd(
        ptr(q2), S if q_rows_total is None else q_rows_total, q2.stride(0), ptr(k2), ptr(v2),
        k2.shape[0], k2.stride(0), ptr(out), out.stride(0), num_heads, D, ptr(plan.q_pairs),
        n_pairs, ptr(plan.kv_tiles), ptr(plan.row_masks), ptr(plan.order), scale,
        ptr(_dev_err(q2.device)), stream_ptr(q2.device)))
    return out


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
    q, k = hier_prep_qk(qx, kx, freqs, num_heads, norm_q_weight=norm_q_weight,
                        norm_k_weight=norm_k_weight, cam_tokens=cam_tokens,
                        cam_q_weight=cam_q_weight, cam_k_weight=cam_k_weight, eps=eps)
    return attention_from_plan(q, k, v, block_mask, num_heads, out=out)


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

    ``mask`` is the :class:`HierBlockMask` returned by
    ``multics_b200.hier_masks.build_stage2_hier_flex_block_mask`` (the
    reference passes a dense bool mask or a Flex BlockMask).  The q/k/v/o
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

    def project_qkv(self, x, freqs, cam_tokens=None):
        """Projected + fused-prologue ``(q, k, v)`` as ``[S, dim]`` bf16 rows."""
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
            cam_k_weight=None if self.cam_k is None else self.cam_k.weight, eps=self.norm_q.eps)
        return q, k, _rows(v)

    def forward(self, x, freqs, mask=None, cam_tokens=None):
        if not isinstance(mask, HierBlockMask):
            raise TypeError("multics_b200 SelfAttention.forward requires a HierBlockMask "
                            "(build_stage2_hier_flex_block_mask)")
        q, k, v = self.project_qkv(x, freqs, cam_tokens)
        out = attention_from_plan(q, k, v, mask, self.num_heads)
        return self.o(out.unsqueeze(0))

"""Training path of the hierarchical attention on B200: autograd over the
128x128 block plan.

The reference trains its hierarchical self-attention with FlexAttention
over the grouping's BlockMask (``multics/models/attention.py:322-353``;
``forward_hier_tiled_ste`` keeps the Flex Jacobian, ``:367-434``).  Here the
forward is the tcgen05 attention kernel run on the block plan with its
log2-sum-exp kept, and the backward is three kernels
(``csrc/hier_bwd.cu``): Delta = rowsum(dO * O), dQ over the forward's
query-major plan, dK and dV over its key-major transpose.  The camera add,
RMSNorm and RoPE before it run as the fused prologue kernel with its own
backward kernel (:func:`prologue_grad`).

:func:`hier_block_attention_grad` is the differentiable attention;
:meth:`multics_b200.attention.SelfAttention.forward` uses it whenever autograd
is recording.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr
from .attention import _dev_err, _rows
from .hier_masks import HierBlockMask

__all__ = ["BlockPlanGrad", "block_plan_grad", "hier_block_attention_grad", "plan_attention_grad",
           "prologue_grad"]


def _plan_extent(plan):
    """(references of key blocks by query tiles at most, row masks) of a plan."""
    if isinstance(plan, HierBlockMask):
        return plan.n_partial + plan.n_full, (plan.row_masks.shape[0] if plan.n_partial > 0 else 0)
    return 2 * plan.kv_tiles.shape[0], plan.row_masks.shape[0]


class BlockPlanGrad:
    """Key-major form of a 128-aligned plan (``hier_bwd_plan_transpose``): per
    key block the query tiles that see it and per-key-row masks.  ``plan`` is
    a :class:`HierBlockMask` or any plan whose query tiles start on multiples
    of 128 rows and whose key tiles are 128-row blocks (an aligned
    :class:`~multics_b200.action.SharedMaskPlan`)."""

    def __init__(self, plan, kv_rows: int):
        dev = plan.q_pairs.device
        self.n_kb = (kv_rows + 127) // 128
        capacity, n_masks = _plan_extent(plan)
        i32 = dict(dtype=torch.int32, device=dev)
        ws = torch.empty(2 * self.n_kb, **i32)
        self.k_off = torch.empty(self.n_kb + 1, **i32)
        self.k_ent = torch.empty((max(capacity, 1), 4), **i32)
        self.t_masks = torch.empty((max(n_masks, 1), 128, 4), **i32)
        status = torch.empty(1, **i32)
        check(_lib.lib().hier_bwd_plan_transpose(
            ptr(plan.q_pairs), plan.q_pairs.shape[0], ptr(plan.kv_tiles), ptr(plan.row_masks),
            n_masks, self.n_kb, ptr(ws), ptr(self.k_off), ptr(self.k_ent), capacity,
            ptr(self.t_masks), ptr(status), stream_ptr(dev)))
        st = int(status.item())
        if st & 1:
            raise NotImplementedError(
                "the attention backward needs a plan of 128-aligned query and key tiles over "
                "one key stream (a block plan, or an aligned shared-mask plan)")
        if st & 2:
            raise RuntimeError("key-major plan exceeded its capacity")


def block_plan_grad(plan, kv_rows: int) -> BlockPlanGrad:
    """The key-major plan of ``plan``, built once per plan (kept on it)."""
    gp = getattr(plan, "_grad_plan", None)
    if gp is None or gp.n_kb != (kv_rows + 127) // 128:
        gp = BlockPlanGrad(plan, kv_rows)
        object.__setattr__(plan, "_grad_plan", gp)
    return gp


def _sequence_plan_for(plan, num_heads, scale, D, q_rows, kv_rows):
    """The sequence plan of a block mask's grouping when the forward can run
    on it (self-attention at the default softmax scale), else None."""
    if not isinstance(plan, HierBlockMask) or q_rows != kv_rows or q_rows != plan.S:
        return None
    if abs(scale - 1.0 / math.sqrt(D)) > 1e-9 * scale:
        return None
    from .attention import sequence_plan

    return sequence_plan(plan, num_heads)


class _PlanAttention(torch.autograd.Function):
    """Attention of query rows ``[Sq, H*D]`` over key/value rows ``[Sk, H*D]``
    under an aligned plan; forward keeps the log2-sum-exp for the backward.
    For a block mask whose grouping has a sequence plan the forward runs on
    that plan (the backward only needs O and the log2-sum-exp, whichever
    plan produced them)."""

    @staticmethod
    def forward(ctx, q, k, v, plan, num_heads, scale):
        q2, k2, v2 = (_rows(t).contiguous() for t in (q, k, v))
        for name, t in (("q", q2), ("k", k2), ("v", v2)):
            if t.dtype != torch.bfloat16 or not t.is_cuda:
                raise NotImplementedError(f"the B200 attention needs bf16 CUDA {name}")
        if k2.shape != v2.shape or k2.shape[1] != q2.shape[1]:
            raise ValueError(f"q {tuple(q2.shape)}, k {tuple(k2.shape)}, v {tuple(v2.shape)} "
                             f"disagree")
        S, dim = q2.shape
        D = dim // num_heads
        dev = q2.device
        out = torch.empty_like(q2)
        lse = torch.empty((S, num_heads), dtype=torch.float32, device=dev)
        sp = _sequence_plan_for(plan, num_heads, scale, D, S, k2.shape[0])
        if sp is not None:
            # the forward on the grouping's sequence plan (denser tiles than
            # the block plan the backward needs): q and k with the hub rows
            # in the plan's group-major order, out and lse in sequence order
            A = sp.A
            q_plan = torch.cat([q2[:A], q2[A:].index_select(0, sp.hub_src)])
            k_plan = torch.cat([k2[:A], k2[A:].index_select(0, sp.hub_src)])
            sp.attend(q_plan, k_plan, v2, out=out, lse=lse)
            ctx.save_for_backward(q2, k2, v2, out, lse)
            ctx.plan, ctx.num_heads, ctx.scale = plan, num_heads, scale
            ctx.shapes = (q.shape, k.shape, v.shape)
            return out.view(q.shape)
        kp = (ctypes.c_void_p * 1)(k2.data_ptr())
        vp = (ctypes.c_void_p * 1)(v2.data_ptr())
        rows = (ctypes.c_int64 * 1)(k2.shape[0])
        strides = (ctypes.c_int64 * 1)(k2.stride(0))
        check(_lib.lib().hier_attn_fwd_streams(
            ptr(q2), S, q2.stride(0), 1, kp, vp, rows, strides, ptr(out), out.stride(0), None,
            num_heads, D, ptr(plan.q_pairs), plan.q_pairs.shape[0], ptr(plan.kv_tiles),
            ptr(plan.row_masks), 128, ptr(plan.order), scale, ptr(lse), None, ptr(_dev_err(dev)),
            stream_ptr(dev)))
        ctx.save_for_backward(q2, k2, v2, out, lse)
        ctx.plan, ctx.num_heads, ctx.scale = plan, num_heads, scale
        ctx.shapes = (q.shape, k.shape, v.shape)
        return out.view(q.shape)

    @staticmethod
    def backward(ctx, dout):
        q2, k2, v2, out, lse = ctx.saved_tensors
        plan, H, scale = ctx.plan, ctx.num_heads, ctx.scale
        S, dim = q2.shape
        D = dim // H
        dev = q2.device
        do2 = dout.reshape(S, dim).to(torch.bfloat16).contiguous()
        rows_pad = (S + 127) // 128 * 128
        delta = torch.empty((H, rows_pad), dtype=torch.float32, device=dev)
        lse_t = torch.empty_like(delta)
        L = _lib.lib()
        st = stream_ptr(dev)
        err = _dev_err(dev)
        check(L.hier_attn_bwd_prep(ptr(out), out.stride(0), ptr(do2), do2.stride(0), ptr(lse), S,
                                   H, D, ptr(delta), ptr(lse_t), rows_pad, st))
        dq = torch.empty_like(q2)
        dk = torch.empty_like(k2)
        dv = torch.empty_like(v2)
        kv_rows = k2.shape[0]
        check(L.hier_attn_bwd_dq(
            ptr(q2), S, q2.stride(0), ptr(k2), ptr(v2), kv_rows, k2.stride(0), ptr(do2),
            do2.stride(0), ptr(lse_t), ptr(delta), rows_pad, H, D, ptr(plan.q_pairs),
            plan.q_pairs.shape[0], ptr(plan.kv_tiles), ptr(plan.row_masks), 128, scale, ptr(dq),
            dq.stride(0), ptr(err), st))
        gp = block_plan_grad(plan, kv_rows)
        check(L.hier_attn_bwd_dkv(
            ptr(q2), S, q2.stride(0), ptr(k2), ptr(v2), kv_rows, k2.stride(0), ptr(do2),
            do2.stride(0), ptr(lse_t), ptr(delta), rows_pad, H, D, ptr(gp.k_off), ptr(gp.k_ent),
            ptr(gp.t_masks), gp.n_kb, scale, ptr(dk), dk.stride(0), ptr(dv), dv.stride(0),
            ptr(err), st))
        sq, sk, sv = ctx.shapes
        return dq.view(sq), dk.view(sk), dv.view(sv), None, None, None


class _PrologueFn(torch.autograd.Function):
    """camera add + RMSNorm + RoPE of q and k with the fused kernels both ways
    (``hier_prep_qk`` / ``hier_prep_qk_bwd``)."""

    @staticmethod
    def forward(ctx, qx, kx, nqw, nkw, wcq, wck, cam, ft, num_heads, eps):
        from .attention import hier_prep_qk

        q, k = hier_prep_qk(qx, kx, ft, num_heads, norm_q_weight=nqw, norm_k_weight=nkw,
                            cam_tokens=cam, cam_q_weight=wcq, cam_k_weight=wck, eps=eps)
        ctx.save_for_backward(qx, kx, nqw, nkw, wcq, wck, cam, ft)
        ctx.num_heads, ctx.eps = num_heads, eps
        return q, k

    @staticmethod
    def backward(ctx, gq, gk):
        qx, kx, nqw, nkw, wcq, wck, cam, ft = ctx.saved_tensors
        q2, k2 = _rows(qx).contiguous(), _rows(kx).contiguous()
        S, dim = q2.shape
        H = ctx.num_heads
        dev = q2.device
        gq = torch.zeros_like(q2) if gq is None else gq.reshape(S, dim).to(torch.bfloat16).contiguous()
        gk = torch.zeros_like(k2) if gk is None else gk.reshape(S, dim).to(torch.bfloat16).contiguous()
        n = ctypes.c_int32()
        L = _lib.lib()
        check(L.hier_prep_qk_bwd_partials(S, ctypes.byref(n)))
        part = torch.empty((2, n.value, dim), dtype=torch.float32, device=dev)
        dqx, dkx = torch.empty_like(q2), torch.empty_like(k2)
        c2 = None if cam is None else _rows(cam).to(torch.bfloat16).contiguous()
        bf = lambda t: None if t is None else t.to(torch.bfloat16).contiguous()
        wq, wk, nq, nk = bf(wcq), bf(wck), bf(nqw), bf(nkw)
        check(L.hier_prep_qk_bwd(
            ptr(q2), ptr(k2), q2.stride(0), ptr(c2), 0 if c2 is None else c2.shape[1], ptr(wq),
            ptr(wk), ptr(nq), ptr(nk), ptr(ft), ft.shape[0], S, H, dim // H, float(ctx.eps),
            ptr(gq), ptr(gk), gq.stride(0), ptr(dqx), ptr(dkx), dqx.stride(0), ptr(part),
            stream_ptr(dev)))
        dw = part.sum(1)
        dwcq = dwck = None
        if c2 is not None:
            dwcq = (dqx.t() @ c2).to(wcq.dtype)
            dwck = (dkx.t() @ c2).to(wck.dtype)
        return (dqx.view(qx.shape), dkx.view(kx.shape), dw[0].to(nqw.dtype), dw[1].to(nkw.dtype),
                dwcq, dwck, None, None, None, None)


def prologue_grad(qx, kx, freqs, num_heads, *, norm_q_weight, norm_k_weight, cam_tokens=None,
                  cam_q_weight=None, cam_k_weight=None, eps=1e-6):
    """Differentiable ``hier_prep_qk``: roped ``(q, k)`` ``[S, H*D]`` from the
    projections ``qx``, ``kx``, with gradients for them, the norm weights
    and the camera adapters (camera tokens get none)."""
    from .attention import freqs_table

    ft = freqs if (freqs.dtype == torch.float32 and freqs.dim() == 3
                   and freqs.shape[-1] == 2) else freqs_table(freqs)
    ft = ft.to(qx.device).contiguous()
    return _PrologueFn.apply(qx, kx, norm_q_weight, norm_k_weight, cam_q_weight, cam_k_weight,
                             cam_tokens, ft, num_heads, eps)


def hier_block_attention_grad(q, k, v, mask, num_heads: int, *, softmax_scale=None):
    """Differentiable masked attention on the B200 kernels: ``q``, ``k``,
    ``v`` bf16 ``[S, H*128]`` (or ``[1, S, H*128]``), ``mask`` anything
    :meth:`~multics_b200.attention.SelfAttention.forward` accepts (a
    :class:`HierBlockMask`, a dense bool mask, or None).  Always the block
    plan: the gradients need the aligned 128x128 tiles of its key-major
    transpose."""
    from .attention import attention_mask_plan

    S = q.shape[-2]
    bm = mask if isinstance(mask, HierBlockMask) else attention_mask_plan(mask, S, q.device)
    if bm.S != S:
        raise ValueError(f"block mask is for S={bm.S}, got {S} tokens")
    D = q.shape[-1] // num_heads
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    return _PlanAttention.apply(q, k, v, bm, num_heads, scale)


def plan_attention_grad(q, k, v, plan, num_heads: int, *, softmax_scale=None):
    """Differentiable attention of query rows ``q`` ``[Sq, H*128]`` over
    key/value rows ``k``, ``v`` ``[Sk, H*128]`` (bf16) under a 128-aligned
    ``plan`` (a :class:`HierBlockMask` or an aligned
    :class:`~multics_b200.action.SharedMaskPlan`, as the batched action
    attentions use it)."""
    D = q.shape[-1] // num_heads
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    return _PlanAttention.apply(q, k, v, plan, num_heads, scale)

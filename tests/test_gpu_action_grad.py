"""Training backward of the action-branch attentions on the GPU (the DiT
block's per-frame mouse attention and keyboard cross-attention,
``multics/models/blocks.py:677-697``).

* The aligned shared-mask plan gives the same forward as the packed plan.
* dQ, dK, dV of ``shared_mask_attention`` under autograd (aligned plan,
  key-major transpose, tcgen05 backward kernels) match fp32 autograd of the
  batch's block-diagonal masked attention, on temporal, keyboard and random
  masks with rows without keys and keys no query sees.
* At configuration 3's sizes (880 x 42 frames; 4 x 9 240 rows over 504
  keys; 24 heads) on sampled batch entries.
* ``SelfAttention`` over a batch (projections, fused prologue with a RoPE
  table shared by the batch, attention) and ``CrossAttention`` train against
  the fp32 autograd of the reference's module math
  (``oracle.ref_cpu_path.action_temporal_forward`` / ``action_cross_forward``).
Tolerance for a bf16 gradient against fp32: max-abs <= 3e-2 of the
reference's largest magnitude and cosine >= 0.999.  For the module-level
gradients the bound is the larger of that and twice the error of the same
math run by PyTorch in bf16: some parameter gradients are small residuals of
cancelling terms (softmax is shift-invariant, so the key gradients of one
query sum to zero and k's bias gradient is what the RMSNorm leaves of them),
where bf16 arithmetic itself cannot meet 3e-2.
"""

import math

import numpy as np
import pytest
import torch

from oracle import ref_cpu_path as R

pytestmark = pytest.mark.gpu

REL_MAX = 3e-2
MIN_COS = 0.999


def _errs(got, ref):
    got, ref = got.detach().float().cpu(), ref.detach().float().cpu()
    scale = float(ref.abs().max()) + 1e-12
    err = float((got - ref).abs().max()) / scale
    cos = float((got * ref).sum() / (got.norm() * ref.norm() + 1e-30))
    return err, cos


def _check(got, ref, what, base=None):
    """``got`` against the fp32 ``ref``; ``base``: PyTorch's bf16 result of
    the same math, whose own error widens the bound up to twice it."""
    assert torch.isfinite(got.float()).all(), what
    err, cos = _errs(got, ref)
    max_err, min_cos = REL_MAX, MIN_COS
    if base is not None:
        b_err, b_cos = _errs(base, ref)
        max_err = max(max_err, 2 * b_err)
        min_cos = min(min_cos, 1 - 2 * (1 - b_cos))
    assert err <= max_err, (what, err, max_err)
    assert cos >= min_cos, (what, cos, min_cos)


def _bf16_grads(fn, inputs, w, dout):
    """Gradients of ``fn`` run by PyTorch on the CPU in bf16 (inputs, then
    weights by name)."""
    xs = [t.detach().cpu().bfloat16().requires_grad_(True) for t in inputs]
    wb = {n: t.detach().bfloat16().requires_grad_(True) for n, t in w.items()}
    out = fn(*xs, wb)
    out.backward(dout.cpu().bfloat16())
    return out.detach(), [t.grad for t in xs], {n: t.grad for n, t in wb.items()}


def _mask(kind, arg, Lq, Lk):
    if kind == "temporal":
        return R.temporal_block_causal_mask(Lq, *arg)
    if kind == "keyboard":
        n, win, L = arg
        return R.keyboard_mask(R.temporal_block_causal_mask(Lq // L, n, win), L)
    rng = np.random.default_rng(Lq * 7 + Lk)
    m = rng.random((Lq, Lk)) < arg
    m[1] = False      # a query row without keys
    m[:, 2] = False   # a key no query sees
    return m


def _fp32_attention(q, k, v, dense, H):
    """Masked attention in fp32 with autograd over flat rows; a row without
    keys gives 0."""
    Sq, dim = q.shape
    D = dim // H
    qh, kh, vh = (t.view(t.shape[0], H, D).transpose(0, 1) for t in (q, k, v))
    s = (qh @ kh.transpose(1, 2)) / math.sqrt(D)
    s = s.masked_fill(~dense[None], float("-inf"))
    mx = s.amax(-1, keepdim=True).detach()
    mx = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    e = torch.exp(s - mx)
    den = e.sum(-1, keepdim=True)
    p = e / torch.where(den > 0, den, torch.ones_like(den))
    return (p @ vh).transpose(0, 1).reshape(Sq, dim)


CASES = [
    (6, 42, 42, "temporal", (1, -1)),
    (7, 42, 42, "temporal", (7, 24)),
    (3, 9 * 7, 9 * 12, "keyboard", (3, 4, 7)),
    (2, 30 * 11, 30 * 12, "keyboard", (2, -1, 11)),
    (3, 129, 200, "random", 0.3),
    (9, 5, 300, "random", 0.5),
    (4, 200, 17, "random", 0.1),
]


@pytest.mark.parametrize("B,Lq,Lk,kind,arg", CASES)
def test_aligned_plan_forward_matches_packed(B, Lq, Lk, kind, arg):
    from multics_b200.action import shared_mask_attention, shared_mask_plan
    from multics_b200.attention import device_error

    H = 2
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(B, L, H * 128, generator=g, device="cuda").bfloat16()
               for L in (Lq, Lk, Lk))
    m = torch.from_numpy(_mask(kind, arg, Lq, Lk)).cuda()
    packed = shared_mask_attention(q, k, v, H, m)
    plan = shared_mask_plan(m, B, Lq, Lk, "cuda", aligned=True)
    aligned = shared_mask_attention(q, k, v, H, m, plan=plan)
    torch.cuda.synchronize()
    assert device_error() == 0
    err = float((packed.float() - aligned.float()).abs().max())
    assert err <= 1e-2, err


@pytest.mark.parametrize("B,Lq,Lk,kind,arg", CASES)
def test_shared_mask_attention_grads_match_fp32(B, Lq, Lk, kind, arg):
    from multics_b200.action import shared_mask_attention
    from multics_b200.attention import device_error

    dev = torch.device("cuda")
    H = 2
    dim = H * 128
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + Lq)
    q, k, v = (torch.randn(B, L, dim, generator=g, device=dev).mul(0.7).bfloat16()
               .requires_grad_(True) for L in (Lq, Lk, Lk))
    dout = torch.randn(B, Lq, dim, generator=g, device=dev).bfloat16()
    m = torch.from_numpy(_mask(kind, arg, Lq, Lk)).to(dev)
    err0 = device_error(dev)
    out = shared_mask_attention(q, k, v, H, m)
    out.backward(dout)
    torch.cuda.synchronize()
    assert device_error(dev) == err0 == 0
    dense = torch.block_diag(*([m] * B))
    qf, kf, vf = (t.detach().float().reshape(-1, dim).requires_grad_(True) for t in (q, k, v))
    ref = _fp32_attention(qf, kf, vf, dense, H)
    ref.backward(dout.float().reshape(-1, dim))
    _check(out.detach().reshape(-1, dim), ref.detach(), "out")
    _check(q.grad.reshape(-1, dim), qf.grad, "dq")
    _check(k.grad.reshape(-1, dim), kf.grad, "dk")
    _check(v.grad.reshape(-1, dim), vf.grad, "dv")
    empty = ~dense.any(1)
    if bool(empty.any()):
        assert bool((q.grad.reshape(-1, dim)[empty] == 0).all()), "rows without keys: dq = 0"
    unseen = ~dense.any(0)
    if bool(unseen.any()):
        assert bool((k.grad.reshape(-1, dim)[unseen] == 0).all())
        assert bool((v.grad.reshape(-1, dim)[unseen] == 0).all())


def _init(module):
    with torch.no_grad():
        for p in module.parameters():
            p.normal_(0, 0.05)
        module.norm_q.weight.add_(1.0)
        module.norm_k.weight.add_(1.0)
    return {n: p.detach().float().cpu().clone().requires_grad_(True)
            for n, p in module.named_parameters()}


@pytest.mark.parametrize("B,F,n,win", [(6, 42, 1, -1), (5, 42, 7, 24), (3, 21, 3, 6)])
def test_temporal_self_attention_training_matches_fp32(B, F, n, win):
    """The per-frame action attention as a training step: ``SelfAttention``
    over ``B`` frame sequences with autograd (fused prologue forward and
    backward with one RoPE table for the batch, aligned shared-mask plan)."""
    from multics_b200.action import get_temporal_block_causal_mask
    from multics_b200.attention import SelfAttention
    from multics_b200.rope import precompute_freqs_cis

    dev = torch.device("cuda")
    H, D = 2, 128
    torch.manual_seed(B * 100 + F)
    sa = SelfAttention(H * D, H, eps=1e-6).to(dev)
    w = _init(sa)
    sa.to(torch.bfloat16)
    x = torch.randn(B, F, H * D, device=dev).bfloat16().requires_grad_(True)
    freqs = precompute_freqs_cis(D, end=F).unsqueeze(1).to(dev)
    mask = get_temporal_block_causal_mask(F, n, win, device=dev)
    out = sa(x, freqs, mask)
    dout = torch.randn_like(out)
    out.backward(dout)
    torch.cuda.synchronize()
    xr = x.detach().float().cpu().requires_grad_(True)
    mask_np = R.temporal_block_causal_mask(F, n, win)
    ref = R.action_temporal_forward(xr, w, H, mask_np)
    ref.backward(dout.float().cpu())
    b_out, (b_dx,), b_w = _bf16_grads(
        lambda xb, wb: R.action_temporal_forward(xb, wb, H, mask_np), [x], w, dout)
    _check(out.detach(), ref.detach(), "out", b_out)
    _check(x.grad, xr.grad, "dx", b_dx)
    for name, p in sa.named_parameters():
        _check(p.grad, w[name].grad, name, b_w[name])


@pytest.mark.parametrize("P,F,n,win,L", [(2, 6, 1, -1, 11), (3, 7, 3, 4, 20)])
def test_keyboard_cross_attention_training_matches_fp32(P, F, n, win, L):
    """The keyboard cross-attention as a training step: ``CrossAttention``
    with the repeated frame mask, gradients for the queries' tokens, the
    keyboard context and every weight."""
    from multics_b200.action import get_temporal_block_causal_mask, keyboard_frame_mask
    from multics_b200.attention import CrossAttention

    dev = torch.device("cuda")
    H, D, K = 2, 128, 12
    torch.manual_seed(P * 100 + L)
    ca = CrossAttention(H * D, H, eps=1e-6).to(dev)
    w = _init(ca)
    ca.to(torch.bfloat16)
    x = torch.randn(P, F * L, H * D, device=dev).bfloat16().requires_grad_(True)
    ctx = torch.randn(P, F * K, H * D, device=dev).bfloat16().requires_grad_(True)
    mask = keyboard_frame_mask(get_temporal_block_causal_mask(F, n, win, device=dev), L, K)
    out = ca(x, ctx, mask)
    dout = torch.randn_like(out)
    out.backward(dout)
    torch.cuda.synchronize()
    xr = x.detach().float().cpu().requires_grad_(True)
    cr = ctx.detach().float().cpu().requires_grad_(True)
    m = R.keyboard_mask(R.temporal_block_causal_mask(F, n, win), L, K)
    ref = R.action_cross_forward(xr, cr, w, H, m)
    ref.backward(dout.float().cpu())
    b_out, (b_dx, b_dc), b_w = _bf16_grads(
        lambda xb, cb, wb: R.action_cross_forward(xb, cb, wb, H, m), [x, ctx], w, dout)
    _check(out.detach(), ref.detach(), "out", b_out)
    _check(x.grad, xr.grad, "dx", b_dx)
    _check(ctx.grad, cr.grad, "dctx", b_dc)
    for name, p in ca.named_parameters():
        _check(p.grad, w[name].grad, name, b_w[name])


def test_config3_action_backward_full_size():
    """Gradients at configuration 3's sizes, 24 heads: the per-frame attention
    (880 sequences of 42 frames, 1-frame block-causal mask) and the keyboard
    cross-attention (4 players x 9 240 rows over 504 keyboard keys).  A batch
    entry's gradients depend on its own rows only, so sampled entries are
    checked against fp32 autograd."""
    from multics_b200.action import (get_temporal_block_causal_mask, keyboard_frame_mask,
                                     shared_mask_attention)
    from multics_b200.attention import device_error

    dev = torch.device("cuda")
    H = 24
    dim = H * 128
    fm = get_temporal_block_causal_mask(42, 1, -1, device=dev)
    cases = (("temporal", 880, 42, 42, fm, (0, 437, 879)),
             ("keyboard", 4, 42 * 220, 42 * 12, keyboard_frame_mask(fm, 220, 12), (0, 3)))
    for name, B, Lq, Lk, m, sample in cases:
        g = torch.Generator(device="cuda").manual_seed(B)
        q, k, v = (torch.randn(B, L, dim, generator=g, device=dev).mul(0.7).bfloat16()
                   .requires_grad_(True) for L in (Lq, Lk, Lk))
        dout = torch.randn(B, Lq, dim, generator=g, device=dev).bfloat16()
        shared_mask_attention(q, k, v, H, m).backward(dout)
        torch.cuda.synchronize()
        assert device_error(dev) == 0, name
        for b in sample:
            qf, kf, vf = (t[b].detach().float().requires_grad_(True) for t in (q, k, v))
            _fp32_attention(qf, kf, vf, m, H).backward(dout[b].float())
            _check(q.grad[b], qf.grad, (name, b, "dq"))
            _check(k.grad[b], kf.grad, (name, b, "dk"))
            _check(v.grad[b], vf.grad, (name, b, "dv"))
            del qf, kf, vf
        del q, k, v, dout
        torch.cuda.empty_cache()


def test_grads_follow_a_callers_packed_plan():
    """A packed plan passed with ``mask=None`` while autograd records: the
    attention and its gradients follow the plan's own mask (its aligned
    form), not an unmasked plan."""
    from multics_b200.action import shared_mask_attention, shared_mask_plan

    dev = torch.device("cuda")
    B, Lq, Lk, H = 5, 42, 42, 2
    dim = H * 128
    m = torch.from_numpy(_mask("temporal", (7, 24), Lq, Lk)).to(dev)
    plan = shared_mask_plan(m, B, Lq, Lk, dev)
    assert not plan.aligned
    g = torch.Generator(device="cuda").manual_seed(21)
    q, k, v = (torch.randn(B, L, dim, generator=g, device=dev).mul(0.7).bfloat16()
               .requires_grad_(True) for L in (Lq, Lk, Lk))
    dout = torch.randn(B, Lq, dim, generator=g, device=dev).bfloat16()
    out = shared_mask_attention(q, k, v, H, None, plan=plan)
    out.backward(dout)
    torch.cuda.synchronize()
    assert plan.aligned_form().aligned and plan.aligned_form() is plan.aligned_form()
    dense = torch.block_diag(*([m] * B))
    qf, kf, vf = (t.detach().float().reshape(-1, dim).requires_grad_(True) for t in (q, k, v))
    ref = _fp32_attention(qf, kf, vf, dense, H)
    ref.backward(dout.float().reshape(-1, dim))
    _check(out.detach().reshape(-1, dim), ref.detach(), "out")
    _check(q.grad.reshape(-1, dim), qf.grad, "dq")
    _check(k.grad.reshape(-1, dim), kf.grad, "dk")
    _check(v.grad.reshape(-1, dim), vf.grad, "dv")

"""Training backward of the hierarchical attention on the GPU.

* The key-major plan (``hier_bwd_plan_transpose``) re-expands to exactly the
  transpose of the forward plan's mask, and lists every key block's query
  blocks once, in ascending order.
* dQ, dK, dV of :func:`multics_b200.train.hier_block_attention_grad` match a
  PyTorch fp32 autograd restatement of masked attention (rows without keys:
  no contribution) on hierarchical groupings (labels, membership with idle
  hubs, windows), a caller's dense mask with empty rows, and no mask, at
  sequence lengths that are not multiples of 128.
* The fused prologue's backward (``hier_prep_qk_bwd``) matches fp32 autograd
  of camera add + RMSNorm + RoPE, with and without camera tokens, for one
  RoPE row per token and for a table shared by a batch of sequences.
* The whole attention path (fused prologue, attention) reproduces the
  gradients the reference's own autograd recorded (``tests/golden/
  grads.npz``) for its inputs and camera / norm weights.
* ``SelfAttention`` under autograd (projections included) matches an fp32
  copy of the module.
Tolerance for a bf16 gradient against fp32: max-abs <= 3e-2 of the
reference's largest magnitude and cosine >= 0.999.
"""

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import hier_oracle as O

pytestmark = pytest.mark.gpu

REL_MAX = 3e-2
MIN_COS = 0.999
GRADS = np.load(Path(__file__).parent / "golden" / "grads.npz")
NUM = np.load(Path(__file__).parent / "golden" / "numerics.npz")


def _check(got, ref, what):
    got, ref = got.float(), ref.float()
    assert torch.isfinite(got).all(), what
    scale = float(ref.abs().max()) + 1e-12
    err = float((got - ref).abs().max()) / scale
    cos = float((got * ref).sum() / (got.norm() * ref.norm() + 1e-30))
    assert err <= REL_MAX, (what, err)
    assert cos >= MIN_COS, (what, cos)


def _fp32_attention(q, k, v, mask, H):
    """softmax(q k^T / sqrt(D), masked) v per head in fp32 with autograd;
    a row without keys gives 0."""
    S, dim = q.shape
    D = dim // H
    qh, kh, vh = (t.view(t.shape[0], H, D).transpose(0, 1) for t in (q, k, v))
    s = (qh @ kh.transpose(1, 2)) / math.sqrt(D)
    s = s.masked_fill(~mask[None], float("-inf"))
    mx = s.amax(-1, keepdim=True).detach()
    mx = torch.where(torch.isfinite(mx), mx, torch.zeros_like(mx))
    e = torch.exp(s - mx)
    den = e.sum(-1, keepdim=True)
    p = e / torch.where(den > 0, den, torch.ones_like(den))
    return (p @ vh).transpose(0, 1).reshape(S, dim)


def _hier_case(case, dev):
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask

    P, T, L, N, KL, KG, n, win, mode = case
    g = torch.Generator().manual_seed(hash(case) & 0xFFFF)
    if mode == "labels":
        labels = torch.randint(0, N, (T, P), generator=g)
        for t0 in range(0, T, n):
            labels[t0:t0 + n] = labels[t0]
        kw = dict(group_labels=labels.to(dev), active_group=None)
        okw = dict(labels=labels.numpy(), direct=True)
    else:
        mem = torch.rand(T, N, P, generator=g) < 0.4
        go = ~mem.any(1)
        mem[:, N - 1] = False  # an idle slot: inactive local-hub rows
        kw = dict(group_labels=None, active_group=None, membership=mem.to(dev),
                  global_only=go.to(dev))
        okw = dict(membership=mem.numpy(), global_only=go.numpy(), direct=True)
    bm, S, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, n, win, direct_player=True,
                                                 device=dev, **kw)
    dense = torch.from_numpy(O.dense_mask(P, T, L, N, KL, KG, n, win, **okw)).to(dev)
    return bm, dense


HIER_CASES = [
    # P, T, L, N, KL, KG, n, win, mode
    (4, 6, 50, 2, 4, 3, 1, -1, "labels"),
    (4, 6, 50, 2, 4, 3, 3, 4, "labels"),
    (5, 4, 37, 3, 5, 6, 2, 2, "membership"),
    (3, 5, 130, 2, 16, 6, 1, -1, "labels"),
]


def _masks(kind, dev):
    """(block mask or mask argument, dense bool mask) for a case."""
    from multics_b200.attention import attention_mask_plan

    if kind[0] == "hier":
        return _hier_case(kind[1], dev)
    S = kind[1]
    if kind[0] == "dense":
        g = torch.Generator(device="cuda").manual_seed(S)
        m = torch.rand(S, S, generator=g, device="cuda") < 0.35
        m[3] = False      # a query row without keys
        m[:, 5] = False   # a key no query sees
        return attention_mask_plan(m, S, dev), m
    m = torch.ones(S, S, dtype=torch.bool, device=dev)
    return attention_mask_plan(None, S, dev), m


GRAD_CASES = [("hier", c) for c in HIER_CASES] + [("dense", 300), ("dense", 517), ("none", 389)]


def _ids(c):
    return f"{c[0]}-{c[1]}"


@pytest.mark.parametrize("kind", GRAD_CASES, ids=_ids)
def test_transposed_plan_is_the_transpose(kind):
    from multics_b200.train import block_plan_grad
    from test_gpu_kernels import expand_plan

    dev = torch.device("cuda")
    bm, dense = _masks(kind, dev)
    S = bm.S
    gp = block_plan_grad(bm, S)
    fwd = expand_plan(bm)
    off = gp.k_off.cpu().numpy()
    ent = gp.k_ent.cpu().numpy()
    tm = gp.t_masks.cpu().numpy().view(np.uint32)
    cover = np.zeros((S + 128, S + 128), np.int32)
    vis = np.zeros((S + 128, S + 128), bool)
    for kb in range(gp.n_kb):
        lst = ent[off[kb]:off[kb + 1]]
        assert list(lst[:, 3]) == sorted(lst[:, 3]), "ascending query blocks"
        for qs, qn, sel, _ in lst:
            if sel == -1:
                bits = np.ones((128, 128), bool)
            else:
                w = tm[sel]  # [key row][4 words over query rows]
                bits = ((w[:, np.arange(128) // 32] >> (np.arange(128) % 32)) & 1).astype(bool)
            bits = bits[:, :qn]
            k0 = 128 * kb
            cover[k0:k0 + 128, qs:qs + qn] += 1
            vis[k0:k0 + 128, qs:qs + qn] |= bits
    assert cover.max() <= 1
    assert np.array_equal(vis[:S, :S], fwd.T)
    assert np.array_equal(fwd, dense.cpu().numpy())


@pytest.mark.parametrize("kind", GRAD_CASES, ids=_ids)
def test_block_attention_grads_match_fp32(kind):
    from multics_b200.attention import device_error
    from multics_b200.train import hier_block_attention_grad

    dev = torch.device("cuda")
    bm, dense = _masks(kind, dev)
    S, H = bm.S, 2
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn(S, H * 128, generator=g, device=dev).mul(0.7).bfloat16()
               .requires_grad_(True) for _ in range(3))
    dout = torch.randn(S, H * 128, generator=g, device=dev).bfloat16()
    err0 = device_error(dev)
    out = hier_block_attention_grad(q, k, v, bm, H)
    out.backward(dout)
    torch.cuda.synchronize()
    assert device_error(dev) == err0 == 0
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = _fp32_attention(qf, kf, vf, dense, H)
    ref.backward(dout.float())
    _check(out.detach(), ref.detach(), "out")
    _check(q.grad, qf.grad, "dq")
    _check(k.grad, kf.grad, "dk")
    _check(v.grad, vf.grad, "dv")
    empty = ~dense.any(1)
    if bool(empty.any()):
        assert bool((q.grad[empty] == 0).all()), "rows without keys: dq = 0"
    unseen = ~dense.any(0)
    if bool(unseen.any()):
        assert bool((k.grad[unseen] == 0).all()) and bool((v.grad[unseen] == 0).all())


def _bf(a, dev):
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


@pytest.mark.parametrize("name", json.loads(bytes(GRADS["grad_case_names"]).decode()))
def test_attention_path_grads_match_reference(name):
    """camera add -> RMSNorm -> RoPE -> attention with autograd, from the
    reference's recorded inputs, against its recorded gradients."""
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask
    from multics_b200.train import hier_block_attention_grad, prologue_grad

    dev = torch.device("cuda")
    meta = json.loads(bytes(NUM[f"{name}/meta"]).decode())
    H, D, S = meta["H"], meta["D"], meta["S"]
    qx, kx, v = (_bf(NUM[f"{name}/{t}"], dev)[None].requires_grad_(True) for t in ("qx", "kx", "v"))
    cam = _bf(NUM[f"{name}/cam"], dev)[None]
    wcq, wck, nqw, nkw = (_bf(NUM[f"{name}/{t}"], dev).requires_grad_(True)
                          for t in ("wcq", "wck", "nqw", "nkw"))
    fr = torch.from_numpy(NUM[f"{name}/freqs"]).to(dev)
    freqs = torch.complex(fr[..., 0], fr[..., 1]).unsqueeze(1)
    P, T, L, N, KL, KG = (meta[k] for k in ("P", "T", "L", "N", "KL", "KG"))
    labels = torch.from_numpy(NUM[f"{name}/labels"]).to(dev)
    kw = dict(group_labels=labels, active_group=None)
    if meta["membership"]:
        kw = dict(group_labels=None, active_group=None,
                  membership=torch.from_numpy(NUM[f"{name}/membership"]).to(dev),
                  global_only=torch.from_numpy(NUM[f"{name}/global_only"]).to(dev))
    bm, _, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, meta["n"], meta["win"],
                                                 direct_player=True, device=dev, **kw)
    q, k = prologue_grad(qx, kx, freqs, H, norm_q_weight=nqw, norm_k_weight=nkw,
                         cam_tokens=cam, cam_q_weight=wcq, cam_k_weight=wck)
    out = hier_block_attention_grad(q, k, v[0], bm, H)
    out.backward(_bf(GRADS[f"{name}/dout"], dev))
    torch.cuda.synchronize()
    for t, got in (("qx", qx.grad[0]), ("kx", kx.grad[0]), ("v", v.grad[0]), ("wcq", wcq.grad),
                   ("wck", wck.grad), ("nqw", nqw.grad), ("nkw", nkw.grad)):
        _check(got, torch.from_numpy(GRADS[f"{name}/d_{t}"]).to(dev), (name, t))


def test_self_attention_training_matches_fp32_module():
    """Projections + camera + RMSNorm + RoPE + attention + output projection
    under autograd, against the same module in fp32 (PyTorch attention)."""
    from multics_b200.attention import SelfAttention, _rope_torch
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask
    from multics_b200.rope import self_attn_freqs_with_hub

    dev = torch.device("cuda")
    P, T, h, w, N, KL, KG, H = 4, 3, 4, 10, 2, 8, 6, 2
    L = h * w
    dim = H * 128
    torch.manual_seed(0)
    layer = SelfAttention(dim, H).to(dev)
    layer.enable_camera_pose_qk(12, dropout_p=0.0)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0, 0.05)
        layer.norm_q.weight.add_(1.0)
        layer.norm_k.weight.add_(1.0)
    ref = SelfAttention(dim, H).to(dev)
    ref.enable_camera_pose_qk(12, dropout_p=0.0)
    ref.load_state_dict(layer.state_dict())
    layer.to(torch.bfloat16)
    labels = torch.tensor([[0, 0, 1, 1]] * T, device=dev)
    bm, S, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, 1, -1, labels, None, True,
                                                 dev)
    freqs = self_attn_freqs_with_hub(P, T, h, w, N * KL + KG, 128).to(dev)
    x = torch.randn(1, S, dim, device=dev).bfloat16()
    cam = torch.zeros(1, S, 12, device=dev).bfloat16()
    cam[0, :P * T * L] = torch.randn(P * T * L, 12, device=dev).bfloat16()
    xa = x.clone().requires_grad_(True)
    out = layer(xa, freqs, bm, cam)
    dout = torch.randn_like(out)
    out.backward(dout)
    # fp32 module with PyTorch attention on the oracle's dense mask
    dense = torch.from_numpy(O.dense_mask(P, T, L, N, KL, KG, 1, -1,
                                          labels=labels.cpu().numpy(), direct=True)).to(dev)
    xr = x.float().requires_grad_(True)
    qx, kx, v = ref.q(xr), ref.k(xr), ref.v(xr)
    qx = qx + torch.nn.functional.linear(cam.float(), ref.cam_q.weight)
    kx = kx + torch.nn.functional.linear(cam.float(), ref.cam_k.weight)
    q = _rope_torch(ref.norm_q(qx), freqs, H)
    k = _rope_torch(ref.norm_k(kx), freqs, H)
    o = ref.o(_fp32_attention(q[0], k[0], v[0], dense, H))[None]
    o.backward(dout.float())
    torch.cuda.synchronize()
    _check(out.detach(), o.detach(), "out")
    _check(xa.grad, xr.grad, "dx")
    for (n1, p1), (n2, p2) in zip(layer.named_parameters(), ref.named_parameters()):
        assert n1 == n2
        _check(p1.grad, p2.grad, n1)


@pytest.mark.parametrize("S,F,cam", [(1100, 1100, True), (517, 517, False), (42 * 9, 42, False)])
def test_fused_prologue_grads_match_fp32(S, F, cam):
    """hier_prep_qk / hier_prep_qk_bwd through autograd against fp32 autograd
    of the same math (camera add, RMSNorm over the row, RoPE); F < S: one
    table of F rows shared by S / F sequences."""
    from multics_b200.attention import _rope_torch
    from multics_b200.rope import precompute_freqs_cis
    from multics_b200.train import prologue_grad

    dev = torch.device("cuda")
    H, D = 3, 128
    dim = H * D
    g = torch.Generator(device="cuda").manual_seed(S)
    mk = lambda *sh, s=1.0: (torch.randn(*sh, generator=g, device=dev) * s).bfloat16()
    qx, kx = mk(S, dim).requires_grad_(True), mk(S, dim).requires_grad_(True)
    nqw, nkw = (1 + mk(dim, s=0.1)).requires_grad_(True), (1 + mk(dim, s=0.1)).requires_grad_(True)
    c = wcq = wck = None
    if cam:
        c = mk(S, 12)
        c[S // 2:] = 0  # hub rows without a camera
        c[: S // 2] = c[0]  # runs of one camera row
        c[S // 4: S // 2] = mk(12)
        wcq, wck = mk(dim, 12, s=0.05).requires_grad_(True), mk(dim, 12, s=0.05).requires_grad_(True)
    freqs = precompute_freqs_cis(D, end=F).unsqueeze(1).to(dev)
    q, k = prologue_grad(qx, kx, freqs, H, norm_q_weight=nqw, norm_k_weight=nkw, cam_tokens=c,
                         cam_q_weight=wcq, cam_k_weight=wck)
    gq, gk = mk(S, dim), mk(S, dim)
    (q.float() * gq.float()).sum().add_((k.float() * gk.float()).sum()).backward()
    torch.cuda.synchronize()
    leaves = [qx, kx, nqw, nkw] + ([wcq, wck] if cam else [])
    ref = [t.detach().float().requires_grad_(True) for t in leaves]
    fr = freqs.repeat(S // F, 1, 1)

    def path(x, w, wc):
        y = x if wc is None else x + c.float() @ wc.t()
        y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6) * w
        return _rope_torch(y[None], fr, H)[0]

    qr = path(ref[0], ref[2], ref[4] if cam else None)
    kr = path(ref[1], ref[3], ref[5] if cam else None)
    (qr * gq.float()).sum().add_((kr * gk.float()).sum()).backward()
    _check(q.detach(), qr.detach(), "q")
    _check(k.detach(), kr.detach(), "k")
    for name, got, r in zip(("dqx", "dkx", "dnqw", "dnkw", "dwcq", "dwck"), leaves, ref):
        _check(got.grad, r.grad, name)


@pytest.mark.parametrize("case", HIER_CASES[:2] + HIER_CASES[3:], ids=str)
def test_sequence_plan_forward_matches_block_plan_forward(case, monkeypatch):
    """For labels groupings the training forward runs on the sequence plan
    (hub rows' log2-sum-exp from their partials); forcing the block plan
    gives the same output and gradients within rounding."""
    from multics_b200.attention import FULL_SEQUENCE_PLAN_ENV, sequence_plan
    from multics_b200.train import hier_block_attention_grad

    dev = torch.device("cuda")
    bm, _ = _hier_case(case, dev)
    assert sequence_plan(bm, 2) is not None
    S, H = bm.S, 2
    g = torch.Generator(device="cuda").manual_seed(17)
    base = [torch.randn(S, H * 128, generator=g, device=dev).mul(0.7).bfloat16() for _ in range(3)]
    dout = torch.randn(S, H * 128, generator=g, device=dev).bfloat16()
    res = []
    for mode in ("segments", "blocks"):
        monkeypatch.setenv(FULL_SEQUENCE_PLAN_ENV, mode)
        q, k, v = (t.clone().requires_grad_(True) for t in base)
        out = hier_block_attention_grad(q, k, v, bm, H)
        out.backward(dout)
        torch.cuda.synchronize()
        res.append((out.detach(), q.grad, k.grad, v.grad))
    for name, a, b in zip(("out", "dq", "dk", "dv"), res[0], res[1]):
        _check(a, b, name)

"""SelfAttention.forward (the reference's full-sequence entry,
multics/models/attention.py:436-442) end to end: q/k/v projections, camera
adapters, RMSNorm, RoPE, hierarchical attention and the output projection,
against the oracle's fp32 restatement of the same module, with the sequence
plan (labels grouping) and with the 128x128 block plan, and with every mask
form the reference's call sites pass: the Flex-style block mask, the dense
bool mask of build_stage2_hier_self_attn_mask, a foreign dense mask, and
None."""

import numpy as np
import pytest
import torch

from oracle import hier_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


@pytest.mark.parametrize("plan", ["segments", "blocks"])
@pytest.mark.parametrize("n_block,win", [(1, -1), (2, 3)])
def test_selfattention_forward_matches_fp32(plan, n_block, win, monkeypatch):
    from multics_b200.attention import FULL_SEQUENCE_PLAN_ENV, SelfAttention
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask

    monkeypatch.setenv(FULL_SEQUENCE_PLAN_ENV, plan)
    P, T, h, w, N, KL, KG, H, D = 3, 4, 5, 8, 2, 8, 6, 2, 128
    L, dim = h * w, H * D
    S = P * T * L + T * (N * KL + KG)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(21)
    layer = SelfAttention(dim=dim, num_heads=H)
    layer.enable_camera_pose_qk(12)
    with torch.no_grad():
        for lin in (layer.q, layer.k, layer.v, layer.o):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.05)
            lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.05)
        for lin in (layer.cam_q, layer.cam_k):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.05)
        for nrm in (layer.norm_q, layer.norm_k):
            nrm.weight.copy_(1 + 0.02 * torch.randn(dim, generator=g))
    layer = layer.to(dev, torch.bfloat16).eval()  # no camera dropout
    x = torch.randn(1, S, dim, generator=g).to(torch.bfloat16)
    cam = torch.zeros(S, 12)
    cam[:P * T * L] = torch.randn(P * T, 12, generator=g).repeat_interleave(L, 0)
    cam = cam.to(torch.bfloat16)
    labels = np.array([[0, 1, 1], [0, 0, 1], [1, 0, 1], [1, 1, 0]])[:T]
    for t0 in range(0, T, n_block):
        labels[t0:t0 + n_block] = labels[t0]
    freqs = O.self_attn_freqs_with_hub(P, T, h, w, N * KL + KG, D, (12, 32, 42, 42), 10)
    mask, _, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, n_block, win,
                                                   torch.from_numpy(labels).to(dev), None, True,
                                                   dev)
    out = layer(x.to(dev), torch.from_numpy(freqs).float().to(dev), mask, cam.unsqueeze(0).to(dev))
    torch.cuda.synchronize()

    # fp32 restatement: the same bf16 weights and inputs, fp32 arithmetic
    f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    xf = f(x)[0]
    lin = lambda m, a: a @ f(m.weight).T + f(m.bias)  # noqa: E731
    qx, kx, v = lin(layer.q, xf), lin(layer.k, xf), lin(layer.v, xf)
    qr, kr = O.prologue(qx, kx, f(cam), f(layer.cam_q.weight), f(layer.cam_k.weight),
                        f(layer.norm_q.weight), f(layer.norm_k.weight), freqs, H)
    dense = O.dense_mask(P, T, L, N, KL, KG, n_block, win, labels=labels, direct=True)
    attn = O.masked_attention(qr, kr, v, H, lambda a, b: dense[a:b])
    ref = lin(layer.o, attn)
    got = f(out)[0]
    assert np.isfinite(got).all()
    err = float(np.abs(got - ref).max())
    cos = float((got * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err <= MAX_ABS, err
    assert cos >= MIN_COS, cos


def _layer_and_inputs(P, T, h, w, N, KL, KG, H, seed):
    from multics_b200.attention import SelfAttention

    D = 128
    L, dim = h * w, H * D
    S = P * T * L + T * (N * KL + KG)
    g = torch.Generator().manual_seed(seed)
    layer = SelfAttention(dim=dim, num_heads=H)
    layer.enable_camera_pose_qk(12)
    with torch.no_grad():
        for lin in (layer.q, layer.k, layer.v, layer.o):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.05)
            lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.05)
        for lin in (layer.cam_q, layer.cam_k):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.05)
        for nrm in (layer.norm_q, layer.norm_k):
            nrm.weight.copy_(1 + 0.02 * torch.randn(dim, generator=g))
    layer = layer.to("cuda", torch.bfloat16).eval()
    x = torch.randn(1, S, dim, generator=g).to(torch.bfloat16)
    cam = torch.zeros(S, 12)
    cam[:P * T * L] = torch.randn(P * T, 12, generator=g).repeat_interleave(L, 0)
    cam = cam.to(torch.bfloat16)
    freqs = O.self_attn_freqs_with_hub(P, T, h, w, N * KL + KG, D, (12, 32, 42, 42), 10)
    return layer, x, cam, freqs, S


def _fp32_forward(layer, x, cam, freqs, H, dense):
    """Oracle fp32 restatement of the module; ``dense`` None = unmasked.
    Returns the output and the rows that have at least one key."""
    f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    xf = f(x)[0]
    lin = lambda m, a: a @ f(m.weight).T + f(m.bias)  # noqa: E731
    qx, kx, v = lin(layer.q, xf), lin(layer.k, xf), lin(layer.v, xf)
    qr, kr = O.prologue(qx, kx, f(cam), f(layer.cam_q.weight), f(layer.cam_k.weight),
                        f(layer.norm_q.weight), f(layer.norm_k.weight), freqs, H)
    S = xf.shape[0]
    if dense is None:
        dense = np.ones((S, S), bool)
    attn = O.masked_attention(qr, kr, v, H, lambda a, b: dense[a:b])
    return attn, lin(layer.o, attn), dense.any(1)


def _check(got, ref):
    assert np.isfinite(got).all()
    err = float(np.abs(got - ref).max())
    cos = float((got * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err <= MAX_ABS, err
    assert cos >= MIN_COS, cos


def test_selfattention_forward_accepts_every_mask_form():
    """One layer, one grouping: the block mask, the dense mask that carries
    its grouping, the same mask as a plain tensor (block plan from its
    bytes), and the same mask in float (non-zero allows, as mask.to(bool)
    does) all match the fp32 module."""
    from multics_b200.hier_masks import (HierDenseMask, build_stage2_hier_flex_block_mask,
                                         build_stage2_hier_self_attn_mask)

    P, T, h, w, N, KL, KG, H = 3, 4, 5, 8, 2, 8, 6, 2
    layer, x, cam, freqs, S = _layer_and_inputs(P, T, h, w, N, KL, KG, H, seed=5)
    L = h * w
    dev = torch.device("cuda")
    labels = np.array([[0, 1, 1], [0, 0, 1], [1, 0, 1], [1, 1, 0]])
    lab = torch.from_numpy(labels).to(dev)
    dense = O.dense_mask(P, T, L, N, KL, KG, 1, -1, labels=labels, direct=True)
    _, ref, _ = _fp32_forward(layer, x, cam, freqs, H, dense)
    bm, _, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, 1, -1, lab, None, True, dev)
    dm = build_stage2_hier_self_attn_mask(P, T, L, N, KL, KG, 1, -1, lab, None, True, dev)
    assert isinstance(dm, HierDenseMask) and dm.dtype == torch.bool
    assert torch.equal(dm.cpu(), torch.from_numpy(dense))
    plain = torch.from_numpy(dense).to(dev)
    as_float = plain.float().view(1, 1, S, S)
    xd = x.to(dev)
    fd = torch.from_numpy(freqs).float().to(dev)
    cd = cam.unsqueeze(0).to(dev)
    outs = {}
    for name, m in (("block", bm), ("dense_spec", dm), ("plain", plain), ("float", as_float)):
        with torch.no_grad():
            outs[name] = layer(xd, fd, m, cd)
        torch.cuda.synchronize()
        _check(outs[name].float().cpu().numpy()[0], ref)
    # the grouping-carrying mask runs on the grouping's own plan: same bits
    assert torch.equal(outs["block"], outs["dense_spec"])


@pytest.mark.parametrize("shape", [(2, 3, 4, 8, 2, 4, 3, 2), (3, 5, 5, 9, 2, 8, 5, 1)])
def test_selfattention_forward_unmasked(shape):
    """mask=None: every query attends to every key (the reference's unmasked
    flash_attention), including a length that is not a multiple of 128."""
    P, T, h, w, N, KL, KG, H = shape
    layer, x, cam, freqs, S = _layer_and_inputs(P, T, h, w, N, KL, KG, H, seed=9)
    _, ref, _ = _fp32_forward(layer, x, cam, freqs, H, None)
    dev = torch.device("cuda")
    with torch.no_grad():
        out = layer(x.to(dev), torch.from_numpy(freqs).float().to(dev), None,
                    cam.unsqueeze(0).to(dev))
    torch.cuda.synchronize()
    _check(out.float().cpu().numpy()[0], ref)


def test_dense_plan_of_random_mask_with_empty_rows():
    """A foreign random mask with ragged blocks and rows without any key: the
    attention matches fp32 on the rows with keys and writes 0 on the others
    (where SDPA would produce NaN)."""
    from multics_b200.attention import hier_attention_layer
    from multics_b200.hier_masks import build_dense_block_plan

    from test_gpu_kernels import expand_plan

    P, T, h, w, N, KL, KG, H = 2, 3, 6, 7, 2, 4, 3, 2
    layer, x, cam, freqs, S = _layer_and_inputs(P, T, h, w, N, KL, KG, H, seed=13)
    rng = np.random.default_rng(3)
    dense = rng.random((S, S)) < 0.3
    dense[:, 200:330] = True          # full and ragged 128-blocks
    dense[17] = False                 # rows without keys
    dense[S - 1] = False
    dev = torch.device("cuda")
    bm = build_dense_block_plan(torch.from_numpy(dense).to(dev), S)
    assert np.array_equal(expand_plan(bm), dense)
    has = dense.any(1)
    f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    xf = x.to(dev)[0]
    with torch.no_grad():
        qx, kx, v = layer.q(xf), layer.k(xf), layer.v(xf)
    got = hier_attention_layer(qx, kx, v, torch.from_numpy(freqs).float().to(dev),
                               torch.from_numpy(dense).to(dev), H,
                               norm_q_weight=layer.norm_q.weight, norm_k_weight=layer.norm_k.weight,
                               cam_tokens=cam.to(dev), cam_q_weight=layer.cam_q.weight,
                               cam_k_weight=layer.cam_k.weight)
    torch.cuda.synchronize()
    g = f(got)
    assert not g[~has].any()
    # q/k/v projected in bf16 on the GPU here: compare against fp32 attention
    # of the same projections
    qr, kr = O.prologue(f(qx), f(kx), f(cam), f(layer.cam_q.weight), f(layer.cam_k.weight),
                        f(layer.norm_q.weight), f(layer.norm_k.weight), freqs, H)
    ref = O.masked_attention(qr, kr, f(v), H, lambda a, b: dense[a:b])
    _check(g[has], ref[has])

"""SelfAttention.forward (the reference's full-sequence entry,
multics/models/attention.py:436-442) end to end: q/k/v projections, camera
adapters, RMSNorm, RoPE, hierarchical attention and the output projection,
against the oracle's fp32 restatement of the same module, with the sequence
plan (labels grouping) and with the 128x128 block plan."""

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

"""Parity at the benchmark configurations' real sizes.

Configs 2 (S = 38 556), 4 (8 players regrouped every 3 frames, S = 76 860)
and 5 (10 players in groups 3,3,2,2, S = 95 340) run the whole layer through
``hier_attention_layer`` (fused prologue + the sequence plan every full-size
layer uses) on the benchmark's own seeded inputs.  A sample is checked
against an fp32 torch restatement of the reference path on the GPU
(camera add, RMSNorm over the full row, float64 RoPE, masked softmax
attention; ``attention.py:39-54,231-242,307-320``, ``rope.py:248-254``):
the first and the last frame of every player and every hub row, for the
first and the last head, with mask rows from the oracle (the reference's
predicate evaluated at unit scale and expanded; pinned to the reference's
own masks on CPU).  The tolerance is the one of every attention test:
max-abs <= 2e-2 and cosine >= 0.9995 per sampled block.  Plan status and
the kernels' device error word must be 0.
"""

import numpy as np
import pytest
import torch

from oracle.ref_cpu_path import UnitMask

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


def _fp32_prologue(x, cam, w_cam, w_norm, freqs_c, H, eps=1e-6):
    """fp32 camera add + RMSNorm + float64 RoPE of ``x`` ``[S, H*D]`` on the GPU."""
    xf = x.float() + cam.float() @ w_cam.float().t()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w_norm.float()
    S, dim = xf.shape
    xc = torch.view_as_complex(xf.double().reshape(S, H, dim // H // 2, 2).contiguous())
    return torch.view_as_real(xc * freqs_c).reshape(S, dim).float()


def _sample_ranges(cfg):
    A = cfg.P * cfg.T * cfg.L
    out = []
    for p in range(cfg.P):
        base = p * cfg.T * cfg.L
        out.append((f"player{p}/frame0", base, base + cfg.L))
        out.append((f"player{p}/frame{cfg.T - 1}", base + (cfg.T - 1) * cfg.L, base + cfg.T * cfg.L))
    out.append(("hub rows", A, cfg.S))
    return out


@pytest.mark.parametrize("name", ["cfg2", "cfg4", "cfg5"])
def test_full_size_layer_matches_fp32(name):
    from multics_b200.attention import device_error, hier_attention_layer, sequence_plan
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask, clear_block_mask_cache
    from multics_b200.synth import CONFIGS, make_inputs

    cfg = CONFIGS[name]
    dev = torch.device("cuda")
    inp = make_inputs(cfg, device=dev)
    clear_block_mask_cache()
    bm, S, _ = build_stage2_hier_flex_block_mask(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG,
                                                 cfg.n_block, cfg.local_attn, inp.labels, None,
                                                 cfg.direct, dev)
    assert S == cfg.S
    sp = sequence_plan(bm, cfg.H)
    assert sp is not None, "full-size labels groupings run on the sequence plan"
    assert int(sp.core.status.item()) == 0
    err0 = device_error(dev)
    out = hier_attention_layer(inp.qx, inp.kx, inp.v, inp.freqs, bm, cfg.H,
                               norm_q_weight=inp.nqw, norm_k_weight=inp.nkw,
                               cam_tokens=inp.cam, cam_q_weight=inp.wcq, cam_k_weight=inp.wck)
    torch.cuda.synchronize()
    assert device_error(dev) == err0 == 0
    assert torch.isfinite(out).all()

    # fp32 reference of two heads over the sampled rows
    D, H = cfg.D, cfg.H
    freqs_c = inp.freqs.reshape(S, 1, D // 2).to(dev)
    q32 = _fp32_prologue(inp.qx, inp.cam, inp.wcq, inp.nqw, freqs_c, H)
    k32 = _fp32_prologue(inp.kx, inp.cam, inp.wck, inp.nkw, freqs_c, H)
    v32 = inp.v.float()
    labels = inp.labels.cpu().numpy()
    um = UnitMask(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG, cfg.n_block, cfg.local_attn,
                  labels=labels, direct=cfg.direct)
    scale = 1.0 / np.sqrt(D)
    worst = (0.0, 1.0)
    for label, r0, r1 in _sample_ranges(cfg):
        m = torch.from_numpy(um.rows(r0, r1)).to(dev)
        assert bool(m.any(1).all()), "every sampled row has keys"
        for h in (0, H - 1):
            cols = slice(h * D, (h + 1) * D)
            s = (q32[r0:r1, cols] @ k32[:, cols].t()) * scale
            s = s.masked_fill(~m, float("-inf"))
            ref = torch.softmax(s, -1) @ v32[:, cols]
            got = out[r0:r1, cols].float()
            err = float((got - ref).abs().max())
            cos = float((got * ref).sum() / (got.norm() * ref.norm()))
            worst = (max(worst[0], err), min(worst[1], cos))
            assert err <= MAX_ABS, (label, h, err)
            assert cos >= MIN_COS, (label, h, cos)
    print(f"{name}: S={S} worst max_abs={worst[0]:.3g} cos={worst[1]:.6f}")


def test_full_size_config5_paged():
    """Configuration 5 with its 64-token pages shuffled by seed: the paged
    sequence plan at full size against the same fp32 reference samples."""
    from multics_b200.attention import HierSequencePlan, device_error, freqs_table, hier_prep_qk
    from multics_b200.hier_masks import make_grouping_spec
    from multics_b200.synth import CONFIGS, make_inputs, page_table

    cfg = CONFIGS["cfg5"]
    dev = torch.device("cuda")
    inp = make_inputs(cfg, device=dev)
    spec = make_grouping_spec(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG, cfg.n_block,
                              cfg.local_attn, inp.labels, None, cfg.direct, dev)
    sp = HierSequencePlan(spec, cfg.H, page_table=page_table(cfg))
    assert int(sp.core.status.item()) == 0
    S = cfg.S
    q_plan = torch.empty(S, cfg.dim, dtype=torch.bfloat16, device=dev)
    k_pool = torch.empty(sp.pool_size, cfg.dim, dtype=torch.bfloat16, device=dev)
    err0 = device_error(dev)
    hier_prep_qk(inp.qx, inp.kx, freqs_table(inp.freqs), cfg.H, norm_q_weight=inp.nqw,
                 norm_k_weight=inp.nkw, cam_tokens=inp.cam, cam_q_weight=inp.wcq,
                 cam_k_weight=inp.wck, out=(q_plan, k_pool), out_rows=sp.seq_to_plan,
                 k_out_rows=sp.pool_rows)
    out = sp.attend_paged(q_plan, k_pool, sp.to_pool(inp.v))
    torch.cuda.synchronize()
    assert device_error(dev) == err0 == 0
    D, H = cfg.D, cfg.H
    freqs_c = inp.freqs.reshape(S, 1, D // 2).to(dev)
    q32 = _fp32_prologue(inp.qx, inp.cam, inp.wcq, inp.nqw, freqs_c, H)
    k32 = _fp32_prologue(inp.kx, inp.cam, inp.wck, inp.nkw, freqs_c, H)
    v32 = inp.v.float()
    um = UnitMask(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG, cfg.n_block, cfg.local_attn,
                  labels=inp.labels.cpu().numpy(), direct=cfg.direct)
    scale = 1.0 / np.sqrt(D)
    for label, r0, r1 in _sample_ranges(cfg)[::3] + [_sample_ranges(cfg)[-1]]:
        m = torch.from_numpy(um.rows(r0, r1)).to(dev)
        for h in (0, H - 1):
            cols = slice(h * D, (h + 1) * D)
            s = (q32[r0:r1, cols] @ k32[:, cols].t()) * scale
            ref = torch.softmax(s.masked_fill(~m, float("-inf")), -1) @ v32[:, cols]
            got = out[r0:r1, cols].float()
            err = float((got - ref).abs().max())
            cos = float((got * ref).sum() / (got.norm() * ref.norm()))
            assert err <= MAX_ABS, (label, h, err)
            assert cos >= MIN_COS, (label, h, cos)

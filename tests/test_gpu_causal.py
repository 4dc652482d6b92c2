"""Cached forward (``SelfAttention.causal_forward_hier_hub``) block after block
against the reference's own run recorded in ``golden/causal.npz``: outputs of
every block, and the rolling caches after the last block (indices and local
activity exactly; keys/values to bf16 rounding, since the reference rotates
in float64 and projects on the CPU)."""

import numpy as np
import pytest
import torch

from helpers import golden, jload

pytestmark = pytest.mark.gpu


def _bf16(a):
    return torch.from_numpy(np.asarray(a, np.uint16).astype(np.int16)).view(torch.bfloat16)


def _names():
    return jload(golden("causal")["causal_case_names"])


def _rel_l2(a, b):
    a, b = a.float().flatten(), b.float().flatten()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


@pytest.mark.parametrize("name", _names())
def test_causal_forward_matches_reference(name):
    from multics_b200.attention import SelfAttention
    from multics_b200.kv_cache import new_hier_cache

    g = golden("causal")
    m = jload(g[f"{name}/meta"])
    P, N, L, KL, KG, n, H = (m[k] for k in ("P", "N", "L", "KL", "KG", "n", "heads"))
    D, dim = 128, m["heads"] * 128
    dev = torch.device("cuda")
    layer = SelfAttention(dim=dim, num_heads=H)
    if m["cam"]:
        layer.enable_camera_pose_qk(12, dropout_p=0.0)
    layer = layer.to(device=dev, dtype=torch.bfloat16).eval()
    sd = {}
    for key in layer.state_dict():
        gk = f"{name}/w/{key}" if f"{name}/w/{key}" in g else f"w/{key}"
        sd[key] = _bf16(g[gk]).reshape(layer.state_dict()[key].shape)
    layer.load_state_dict(sd)
    layer.num_frame_per_block = m["n_block"]
    layer.local_attn_size = m["local_attn"]
    if m["no_local"]:
        layer.hier_no_local_hub = True
    cache = new_hier_cache(num_players=P, num_groups=N, num_local_hub_tokens=KL,
                           num_global_hub_tokens=KG, frame_seq_length=L,
                           retention_frames=m["retention"], heads=H, head_dim=D,
                           dtype=torch.bfloat16, device=dev, no_local=m["no_local"])
    mem = go = None
    if m["membership"]:
        mem = torch.from_numpy(g[f"{name}/membership"]).bool().to(dev)
        go = torch.from_numpy(g[f"{name}/global_only"]).bool().to(dev)
    worst = 0.0
    with torch.inference_mode():
        for blk in range(m["blocks"]):
            x = _bf16(g[f"{name}/{blk}/x"]).to(dev)[None]
            freqs = torch.from_numpy(g[f"{name}/{blk}/freqs"]).to(dev)
            cam = None
            if m["cam"]:
                cam = _bf16(g[f"{name}/{blk}/cam"]).to(dev)[None]
            kw = dict(current_start=blk * n * P * L, num_frames=n, num_players=P,
                      num_hub_tokens=N * KL + KG, cam_tokens=cam, direct_player=True)
            if m["membership"]:
                kw.update(membership=mem, global_only=go, active_group=None)
            else:
                kw.update(group_labels=torch.from_numpy(g[f"{name}/{blk}/labels"]).to(dev),
                          active_group=torch.from_numpy(g[f"{name}/{blk}/active"]).bool().to(dev))
            y = layer.causal_forward_hier_hub(x, freqs, cache, **kw)
            ref = _bf16(g[f"{name}/{blk}/out"]).to(dev)
            assert torch.isfinite(y).all()
            r = _rel_l2(y[0], ref)
            worst = max(worst, r)
            assert r < 0.01, (blk, r)
    streams = cache["agent_caches"] + cache["local_hubs"] + [cache["global_hub"]]
    assert len(streams) == m["n_streams"]
    for i, st in enumerate(streams):
        idx = [int(st["global_end_index"]), int(st["local_end_index"])]
        assert idx == g[f"{name}/cache/{i}/idx"].tolist(), i
        for key in ("k", "v"):  # whole buffers: rows past local_end hold evicted data alike
            ref = _bf16(g[f"{name}/cache/{i}/{key}"]).to(dev)
            got = st[key][0]
            assert got.shape == ref.shape
            if ref.any():
                assert _rel_l2(got, ref) < 0.01, (i, key)
            else:
                assert not got.any(), (i, key)
        if f"{name}/cache/{i}/active" in g:
            assert np.array_equal(st["active"].cpu().numpy().astype(np.uint8),
                                  g[f"{name}/cache/{i}/active"]), i

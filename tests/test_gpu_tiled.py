"""Tiled128 layouts on the GPU: device builders bit-exact against the
reference's own layouts, and the tiled attention entry points against the
oracle's masked fp32 attention."""

import numpy as np
import pytest
import torch

from helpers import case_names, tiled_case
from oracle import hier_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


def _full_layouts(meta, dev="cuda"):
    from multics_b200 import tiled as TL

    return TL.build_hier_tiled_full_sequence_layouts(
        device=dev, num_players=meta["P"], num_frames=meta["T"], num_patches=meta["L"],
        num_groups=meta["N"], num_local_hub_tokens=meta["KL"],
        num_global_hub_tokens=meta["KG"], num_frame_per_block=meta["n"],
        local_attn_size=meta["win"], group_labels=torch.tensor(meta["labels"]),
        active_group=torch.tensor(meta["active"], dtype=torch.bool),
        direct_player=meta["direct"])


def _cached_layout(meta, dev="cuda"):
    from multics_b200 import tiled as TL

    t = lambda x: tuple(tuple(r) for r in x)  # noqa: E731
    return TL.build_hier_tiled_cached_layout(
        device=dev, P=meta["P"], N=meta["N"], L=meta["L"], KL=meta["KL"], KG=meta["KG"],
        n_frames=meta["n_frames"], n_block=meta["n_block"], local_attn=meta["local_attn"],
        agent_frame_lists=t(meta["agent"]), local_frame_lists=t(meta["local"]),
        global_frame_list=tuple(meta["glob"]), local_active_frames=t(meta["local_active"]),
        labels=t(meta["labels"]), q_active=t(meta["q_active"]), direct_player=meta["direct"])


@pytest.mark.parametrize("name", case_names("tiled"))
def test_device_tiled_layouts_match_reference(name):
    from multics_b200 import tiled as TL

    TL.clear_hier_tiled_layout_cache()
    meta, ref = tiled_case(name)
    got = _full_layouts(meta) if name.startswith("full") else (_cached_layout(meta),)
    assert len(got) == len(ref)
    for g, r in zip(got, ref):
        for key in ("prog_qbase", "prog_nq", "prog_seg", "kv_index", "kv_count"):
            t = getattr(g, key)
            assert t.dtype == torch.int32, key
            assert np.array_equal(t.cpu().numpy(), r[key]), key
        assert g.kv_valid.dtype == torch.uint8
        assert np.array_equal(g.kv_valid.cpu().numpy(), r["kv_valid"])
        assert [g.logical_slots, g.physical_slots, g.dense_slots] == r["slots"].tolist()


def _full_inputs(meta, H, seed):
    P, T, L, N, KL, KG = (meta[k] for k in ("P", "T", "L", "N", "KL", "KG"))
    S = P * T * L + T * (N * KL + KG)
    g = torch.Generator().manual_seed(seed)
    mk = lambda: (torch.randn((1, S, H, 128), generator=g) * 0.5).to(torch.bfloat16)  # noqa: E731
    return mk(), mk(), mk()


def _tiled_reference(meta, q, k, v, H):
    """Rows of each layout segment attend to the valid slots of its kv row."""
    P, T, L, N, KL, KG = (meta[k] for k in ("P", "T", "L", "N", "KL", "KG"))
    lays = O.tiled_full_sequence_layouts(P, T, L, N, KL, KG, meta["n"], meta["win"],
                                         meta["labels"], meta["active"], meta["direct"])
    segs = []
    for lay in lays:
        seen = set()
        for qb, qn, sid in zip(lay.prog_qbase, lay.prog_nq, lay.prog_seg):
            sel = [int(i) for i, ok in zip(lay.kv_index[sid, :lay.kv_count[sid]],
                                           lay.kv_valid[sid, :lay.kv_count[sid]]) if ok]
            segs.append((int(qb), int(qn), sel))
            seen.add(int(sid))
    f = lambda t: t.float().numpy().reshape(-1, H * 128)  # noqa: E731
    return O.segment_attention(f(q), f(k), f(v), H, segs), segs


@pytest.mark.parametrize("name", [n for n in case_names("tiled") if n.startswith("full")])
def test_tiled_full_sequence_attention_matches_oracle(name):
    from multics_b200 import tiled as TL

    meta, _ = tiled_case(name)
    H = 2
    q, k, v = _full_inputs(meta, H, seed=5)
    lays = _full_layouts(meta)
    out = TL.hierarchical_tiled_full_sequence_attention(
        roped_q=q.cuda(), roped_k=k.cuda(), value=v.cuda(), layouts=lays)
    ref, _ = _tiled_reference(meta, q, k, v, H)
    o = out.float().cpu().numpy().reshape(ref.shape)
    assert np.abs(o - ref).max() <= MAX_ABS
    cos = (o * ref).sum() / (np.linalg.norm(o) * np.linalg.norm(ref))
    assert cos >= MIN_COS
    # a subset of the layouts runs only their query rows
    part = TL.hierarchical_tiled_full_sequence_attention(
        roped_q=q.cuda(), roped_k=k.cuda(), value=v.cuda(), layouts=lays[1:2])
    p = part.float().cpu().numpy().reshape(ref.shape)
    rows = np.zeros(ref.shape[0], bool)
    for qb, qn in zip(lays[1].prog_qbase.cpu().tolist(), lays[1].prog_nq.cpu().tolist()):
        rows[qb:qb + qn] = True
    assert not p[~rows].any()
    assert np.abs(p[rows] - o[rows]).max() == 0


def test_tiled_cached_plugin_matches_cached_backend():
    from multics_b200 import cached as C
    from multics_b200 import tiled as TL

    from test_gpu_cached import _plugin_inputs, _released_meta

    meta = _released_meta()
    kw = _plugin_inputs(meta, 2, seed=21, dev="cuda")
    a = C.hierarchical_cached_attention(**kw)
    kw.pop("hier_no_local_hub")
    b = TL.hierarchical_tiled_cached_attention(**kw)
    assert torch.equal(a, b)


def test_query_active_mask():
    from multics_b200 import tiled as TL

    act = torch.tensor([[True, False], [False, True], [True, True]])
    m = TL.build_hier_query_active_mask(active_group=act, num_players=2, num_frames=3,
                                        num_patches=4, num_groups=2, num_local_hub_tokens=3,
                                        num_global_hub_tokens=2, device="cuda",
                                        dtype=torch.float32)
    assert m.shape == (1, 2 * 3 * 4 + 3 * (2 * 3 + 2), 1)
    local = m[0, 24:42, 0].cpu().reshape(3, 2, 3)
    assert torch.equal(local, act.float()[:, :, None].expand(3, 2, 3))
    assert m[0, :24].eq(1).all() and m[0, 42:].eq(1).all()

"""Cached-step path on the GPU: device metadata and varlen plans bit-exact
against the reference's own outputs, and the cached-backend plugin against
the oracle's per-segment fp32 attention."""

import math

import numpy as np
import pytest
import torch

from helpers import case_names, seg_case, seg_kwargs
from oracle import hier_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


def _meta_args(meta):
    t = lambda x: tuple(tuple(r) for r in x)  # noqa: E731
    return dict(P=meta["P"], N=meta["N"], L=meta["L"], KL=meta["KL"], KG=meta["KG"],
                n_frames=meta["n_frames"], n_block=meta["n_block"],
                local_attn=meta["local_attn"], agent_frame_lists=t(meta["agent"]),
                local_frame_lists=t(meta["local"]), global_frame_list=tuple(meta["glob"]),
                local_active_frames=t(meta["local_active"]),
                labels=None if meta["labels"] is None else t(meta["labels"]),
                q_active=t(meta["q_active"]), direct_player=meta["direct"],
                membership=meta["membership"], global_only=meta["global_only"],
                hier_no_local_hub=meta["no_local"])


@pytest.mark.parametrize("name", case_names("seg"))
def test_device_metadata_matches_reference(name):
    from multics_b200 import cached as C

    meta, ref = seg_case(name)
    C.clear_metadata_cache()
    got = C.build_metadata(device="cuda", block_m=meta["block_m"], **_meta_args(meta))
    for i, key in enumerate(("prog_qbase", "prog_nq", "prog_seg", "kv_index", "kv_count")):
        assert got[i].dtype == torch.int32, key
        assert np.array_equal(got[i].cpu().numpy(), ref[key]), key
    assert got[5] == int(ref["logical_pairs"])
    if "plan_q_index" in ref:
        P, N, L, KL, KG, n = (meta[k] for k in ("P", "N", "L", "KL", "KG", "n_frames"))
        S = P * n * L + n * (N * KL + KG)
        plan = C.get_varlen_plan(kv_index=got[3], kv_count=got[4], qbase=got[0], qlen=got[1],
                                 seg_ids=got[2], query_tokens=S)
        for key in ("q_index", "k_index", "cu_q", "cu_k"):
            assert np.array_equal(plan[key].cpu().numpy().astype(np.int64), ref[f"plan_{key}"]), key
        assert plan["q_index"].dtype == torch.int64 and plan["cu_q"].dtype == torch.int32
        assert [plan["max_q"], plan["max_k"], plan["min_k_index"], plan["max_k_index"]] == \
            ref["plan_scalars"].tolist()
        assert np.array_equal(plan["page_indices"].cpu().numpy(), ref["plan_k_index"])


def test_metadata_cache_hit_returns_same_tensors():
    from multics_b200 import cached as C

    meta, _ = seg_case(case_names("seg")[0])
    C.clear_metadata_cache()
    a = C.build_metadata(device="cuda", block_m=meta["block_m"], **_meta_args(meta))
    b = C.build_metadata(device="cuda", block_m=meta["block_m"], **_meta_args(meta))
    assert all(x is y for x, y in zip(a[:5], b[:5]))


def _plugin_inputs(meta, H, seed, dev, token_activity=False, pool_views=False):
    """Per-stream tensors of the plugin signature for a metadata case."""
    g = torch.Generator().manual_seed(seed)
    P, N, L, KL, KG, n = (meta[k] for k in ("P", "N", "L", "KL", "KG", "n_frames"))
    no_local = meta["no_local"]
    dim = H * 128
    S = P * n * L + n * (N * KL + KG)
    fa = len(meta["agent"][0])
    fl = 0 if no_local else len(meta["local"][0])
    fg = len(meta["glob"]) if KG > 0 else 0

    def frames(fr, w):
        return torch.tensor(list(fr), dtype=torch.int64).repeat_interleave(max(w, 1)).to(dev)

    def rnd(rows):
        return (torch.randn((1, rows, dim), generator=g) * 0.5).to(torch.bfloat16).to(dev)

    kw = dict(P=P, N=N, L=L, KL=KL, KG=KG, n_frames=n, n_block=meta["n_block"],
              local_attn=meta["local_attn"], direct_player=meta["direct"],
              hier_no_local_hub=no_local)
    kw["agent_frames"] = [frames(f, L) for f in meta["agent"]]
    if pool_views:
        # caches as row slices of one larger buffer (a paged pool)
        big_k = rnd(P * fa * L + 64)
        big_v = rnd(P * fa * L + 64)
        kw["agent_keys"] = [big_k[:, 32 + p * fa * L: 32 + (p + 1) * fa * L] for p in range(P)]
        kw["agent_vals"] = [big_v[:, 32 + p * fa * L: 32 + (p + 1) * fa * L] for p in range(P)]
    else:
        kw["agent_keys"] = [rnd(fa * L) for _ in range(P)]
        kw["agent_vals"] = [rnd(fa * L) for _ in range(P)]
    if no_local:
        kw.update(local_frames=[], local_keys=[], local_vals=[], local_active_tokens=[])
    else:
        kw["local_frames"] = [frames(f, KL) for f in meta["local"]]
        kw["local_keys"] = [rnd(fl * KL) for _ in range(N)]
        kw["local_vals"] = [rnd(fl * KL) for _ in range(N)]
        acts = []
        for a in meta["local_active"]:
            t = torch.tensor([bool(x) for x in a]).repeat_interleave(KL)
            if token_activity and KL > 1:
                # an active frame needs only one active token (_active_frames)
                t = t.reshape(-1, KL).clone()
                t[:, 1:] = False
                t = t.reshape(-1)
            acts.append(t.to(dev))
        kw["local_active_tokens"] = acts
    kw["global_frames"] = frames(meta["glob"], KG) if KG > 0 else torch.zeros(0, dtype=torch.long,
                                                                             device=dev)
    kw["global_keys"] = rnd(fg * KG)
    kw["global_vals"] = rnd(fg * KG)
    kw["labels"] = (None if meta["labels"] is None
                    else torch.tensor(meta["labels"], dtype=torch.long, device=dev))
    kw["active"] = torch.tensor(meta["q_active"], dtype=torch.bool, device=dev)
    if meta["membership"] is not None:
        kw["membership"] = torch.tensor(meta["membership"], dtype=torch.bool, device=dev)
        kw["global_only"] = torch.tensor(meta["global_only"], dtype=torch.bool, device=dev)
    kw["roped_q"] = (torch.randn((1, S, H, 128), generator=g) * 0.5).to(torch.bfloat16).to(dev)
    return kw


def _oracle_out(meta, kw, H):
    segs = O.segment_key_lists(**seg_kwargs(meta))
    f = lambda t: t.float().cpu().numpy().reshape(-1, H * 128)  # noqa: E731
    keys = list(kw["agent_keys"]) + list(kw["local_keys"]) + [kw["global_keys"]]
    vals = list(kw["agent_vals"]) + list(kw["local_vals"]) + [kw["global_vals"]]
    kp = np.concatenate([f(k) for k in keys])
    vp = np.concatenate([f(v) for v in vals])
    q = f(kw["roped_q"])
    return O.segment_attention(q, kp, vp, H, segs), segs


def _check(out, ref, segs):
    o = out.float().cpu().numpy().reshape(ref.shape)
    assert np.isfinite(o).all()
    err = np.abs(o - ref).max()
    cos = (o * ref).sum() / (np.linalg.norm(o) * np.linalg.norm(ref) + 1e-30)
    assert err <= MAX_ABS, err
    assert cos >= MIN_COS, cos
    for q0, ql, sel in segs:  # empty segments are exactly zero
        if not sel:
            assert not o[q0:q0 + ql].any()


@pytest.fixture(params=["packed", "per-segment"])
def pack_mode(request, monkeypatch):
    """Run a cached test with the hub rows packed per group (the default) and
    with one query pair per hub segment."""
    from multics_b200 import cached as C

    monkeypatch.setenv(C.CACHED_PACK_ENV, "1" if request.param == "packed" else "0")
    return request.param


@pytest.mark.parametrize("name", [n for n in case_names("seg") if n.endswith("/tile")])
def test_cached_attention_matches_oracle(name, pack_mode):
    from multics_b200 import cached as C

    meta, _ = seg_case(name)
    H = 2
    kw = _plugin_inputs(meta, H, seed=7, dev="cuda")
    out = C.hierarchical_cached_attention(sync_checks=True, **kw)
    assert out.shape == (1, kw["roped_q"].shape[1], H * 128) and out.dtype == torch.bfloat16
    ref, segs = _oracle_out(meta, kw, H)
    _check(out, ref, segs)


def _released_meta(KL=16, inactive_q=False):
    fr = list(range(24))
    return dict(P=4, N=2, L=220, KL=KL, KG=6, n_frames=3, n_block=3, local_attn=21,
                agent=[fr] * 4, local=[fr] * 2, glob=fr,
                local_active=[[True] * 24, [f % 5 != 1 for f in fr]],
                labels=[[0, 0, 1, 1]] * 3,
                q_active=[[True, not inactive_q]] * 3, direct=True, membership=None,
                global_only=None, no_local=False)


@pytest.mark.parametrize("variant", ["released", "inactive_hub", "token_activity", "pool_views"])
def test_cached_attention_released_shape(variant, pack_mode):
    """P=4, L=220 (11x20 patches), 24 retained frames, window 21, n=3."""
    from multics_b200 import cached as C

    meta = _released_meta(inactive_q=variant == "inactive_hub")
    H = 2
    kw = _plugin_inputs(meta, H, seed=11, dev="cuda", token_activity=variant == "token_activity",
                        pool_views=variant == "pool_views")
    out = C.hierarchical_cached_attention(sync_checks=True, **kw)
    ref, segs = _oracle_out(meta, kw, H)
    _check(out, ref, segs)


def test_cached_attention_membership_released_shape(pack_mode):
    from multics_b200 import cached as C

    T = 24
    mem = [[[False] * 4 for _ in range(2)] for _ in range(T)]
    for t in range(T):
        mem[t][0][0] = mem[t][0][1] = True
        mem[t][1][1] = mem[t][1][2] = True  # player 1 anchors both groups
    go = [[False, False, False, True] for _ in range(T)]
    meta = dict(_released_meta(), labels=None, membership=mem, global_only=go)
    H = 2
    kw = _plugin_inputs(meta, H, seed=13, dev="cuda")
    out = C.hierarchical_cached_attention(sync_checks=True, **kw)
    ref, segs = _oracle_out(meta, kw, H)
    _check(out, ref, segs)


def test_cached_attention_is_deterministic_and_leaves_caches():
    from multics_b200 import cached as C

    meta = _released_meta()
    kw = _plugin_inputs(meta, 2, seed=3, dev="cuda")
    before = [k.clone() for k in kw["agent_keys"]]
    a = C.hierarchical_cached_attention(**kw)
    b = C.hierarchical_cached_attention(**kw)
    assert torch.equal(a, b)
    assert all(torch.equal(x, y) for x, y in zip(before, kw["agent_keys"]))


def test_cached_membership_frame_out_of_range_raises():
    from multics_b200 import cached as C

    meta = dict(_released_meta(), labels=None,
                membership=[[[True, True, False, False], [False, False, True, True]]] * 4,
                global_only=[[False] * 4] * 4)
    kw = _plugin_inputs(meta, 1, seed=5, dev="cuda")
    with pytest.raises(IndexError):
        C.hierarchical_cached_attention(sync_checks=True, **kw)


def test_packed_plan_structure():
    """Released shape: 12 player pairs + one pack per group (48 rows) + the
    global pack (18 rows), 128-row masks, rows read from the second query
    block and mapped back to the hub rows."""
    from multics_b200 import cached as C

    meta = _released_meta()
    kw = _plugin_inputs(meta, 2, seed=3, dev="cuda")
    agent = [f.reshape(-1) for f in kw["agent_frames"]]
    local = [f.reshape(-1) for f in kw["local_frames"]]
    g = C._Grouping(P=4, N=2, L=220, KL=16, KG=6, n_frames=3, n_block=3, local_attn=21,
                    direct=True, no_local=False, agent_frames=agent, local_frames=local,
                    local_active=[t.view(torch.uint8) for t in kw["local_active_tokens"]],
                    global_frames=kw["global_frames"].reshape(-1), labels=kw["labels"],
                    q_active=kw["active"].view(torch.uint8), membership=None, global_only=None)
    plan = C.build_cached_plan(g, torch.device("cuda"), pack=True)
    flat = C.build_cached_plan(g, torch.device("cuda"), pack=False)
    qp = plan.q_pairs[:plan.n_pairs].cpu().numpy()
    assert plan.n_pairs == 15 and flat.n_pairs == 21
    S = 4 * 3 * 220 + 3 * (2 * 16 + 6)
    assert [tuple(r[:4]) for r in qp[12:]] == [(S, 48, S, 0), (S + 48, 48, S + 48, 0),
                                               (S + 96, 18, S + 96, 0)]
    assert (qp[12:, 6] == 1).all()
    rows = plan.out_rows.cpu().numpy()
    assert (rows[:S] == np.arange(S)).all()
    aq = 4 * 3 * 220
    assert rows[S:S + 3].tolist() == [aq, aq + 1, aq + 2]            # group 0, frame 0
    assert rows[S + 16] == aq + 2 * 16                               # group 0, frame 1
    assert rows[S + 48] == aq + 16                                   # group 1, frame 0
    assert rows[S + 96] == aq + 3 * 2 * 16                           # global, frame 0
    # a pack of one group has about the tiles of one of its segments
    fq = flat.q_pairs.cpu().numpy()
    seg_tiles = fq[12:18, 5] - fq[12:18, 4]
    pack_tiles = qp[12:14, 5] - qp[12:14, 4]
    assert pack_tiles.max() <= seg_tiles.max() + 2

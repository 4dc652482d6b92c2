"""Pin the CPU oracle against fixtures generated from the reference itself.

Every function of ``oracle/hier_oracle.py`` is compared with the reference's
own outputs recorded by ``tests/golden/gen_golden.py``: bit-exact for masks,
block lists, segment metadata, varlen plans and tiled layouts; fp32-close for
the numerics.
"""

import numpy as np
import pytest

from helpers import (case_names, mask_case, mask_kwargs, num_case, seg_case, seg_kwargs,
                     tiled_case)
from oracle import hier_oracle as O


@pytest.mark.parametrize("name", case_names("mask"))
def test_dense_mask_matches_reference(name):
    c = mask_case(name)
    m = O.dense_mask(c["P"], c["T"], c["L"], c["N"], c["KL"], c["KG"], c["n"], c["win"],
                     **mask_kwargs(c))
    assert m.shape == c["dense"].shape
    assert np.array_equal(m, c["dense"])


@pytest.mark.parametrize("name", case_names("mask"))
def test_flex_block_lists_match_reference(name):
    c = mask_case(name)
    kvn, kvi, fn, fi = O.flex_block_lists(c["dense"], c["S_pad"])
    assert np.array_equal(kvn, c["kv_num_blocks"])
    assert np.array_equal(kvi, c["kv_indices"])
    assert np.array_equal(fn, c["full_kv_num_blocks"])
    assert np.array_equal(fi, c["full_kv_indices"])


def test_logical_pairs_matches_dense_popcount():
    c = mask_case("cfg1_n1")
    pairs = O.logical_pairs(c["P"], c["T"], c["L"], c["N"], c["KL"], c["KG"], c["n"], c["win"],
                            **mask_kwargs(c))
    assert pairs == int(c["dense"].sum()) == 17496


@pytest.mark.parametrize("name", case_names("seg"))
def test_segmented_metadata_matches_reference(name):
    meta, ref = seg_case(name)
    got = O.segmented_metadata(meta["block_m"], **seg_kwargs(meta))
    for i, key in enumerate(("prog_qbase", "prog_nq", "prog_seg", "kv_index", "kv_count")):
        assert np.array_equal(got[i], ref[key]), key
    assert got[5] == int(ref["logical_pairs"])
    if "plan_q_index" in ref:
        P, N, L, KL, KG, n = (meta[k] for k in ("P", "N", "L", "KL", "KG", "n_frames"))
        S = P * n * L + n * (N * KL + KG)
        plan = O.varlen_plan(*got[:5], query_tokens=S)
        for key in ("q_index", "k_index", "cu_q", "cu_k"):
            assert np.array_equal(plan[key], ref[f"plan_{key}"]), key
        assert [plan["max_q"], plan["max_k"], plan["min_k_index"], plan["max_k_index"]] == \
            ref["plan_scalars"].tolist()


@pytest.mark.parametrize("name", case_names("tiled"))
def test_tiled_layouts_match_reference(name):
    meta, lays = tiled_case(name)
    if name.startswith("full"):
        got = O.tiled_full_sequence_layouts(meta["P"], meta["T"], meta["L"], meta["N"],
                                            meta["KL"], meta["KG"], meta["n"], meta["win"],
                                            meta["labels"], meta["active"], meta["direct"])
    else:
        kw = seg_kwargs(dict(meta, membership=None, global_only=None, no_local=False))
        kw.pop("membership")
        kw.pop("global_only")
        kw.pop("no_local")
        got = [O.tiled_cached_layout(**kw)]
    assert len(got) == len(lays)
    for g, r in zip(got, lays):
        for key in ("prog_qbase", "prog_nq", "prog_seg", "kv_index", "kv_count", "kv_valid"):
            assert np.array_equal(getattr(g, key), r[key]), key
        assert [g.logical_slots, g.physical_slots, g.dense_slots] == r["slots"].tolist()


@pytest.mark.parametrize("name", case_names("num"))
def test_prologue_and_attention_match_reference(name):
    d = num_case(name)
    m = d["meta"]
    H = m["H"]
    q, k = O.prologue(d["qx"], d["kx"], d["cam"], d["wcq"], d["wck"], d["nqw"], d["nkw"],
                      d["freqs"], H)
    np.testing.assert_allclose(q, d["roped_q"], atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(k, d["roped_k"], atol=2e-5, rtol=1e-5)
    kw = dict(labels=d["labels"], direct=True)
    if m["membership"]:
        kw = dict(membership=d["membership"], global_only=d["global_only"], direct=True)
    mask = O.dense_mask(m["P"], m["T"], m["L"], m["N"], m["KL"], m["KG"], m["n"], m["win"], **kw)
    assert int(mask.sum()) == int(d["mask_popcount"])
    out = O.masked_attention(q, k, d["v"], H, lambda a, b: mask[a:b])
    np.testing.assert_allclose(out, d["out"], atol=2e-5, rtol=1e-4)


@pytest.mark.parametrize("name", case_names("num"))
def test_rope_tables_match_reference(name):
    d = num_case(name)
    m = d["meta"]
    f = O.self_attn_freqs_with_hub(m["P"], m["T"], m["h"], m["w"], m["N"] * m["KL"] + m["KG"],
                                   m["D"], tuple(m["splits"]), m["pool"])
    np.testing.assert_allclose(f, d["freqs"], atol=1e-6, rtol=0)


def test_oracle_rejects_bad_labels():
    with pytest.raises(ValueError, match=r"must be in \[0,2\)"):
        O.dense_mask(4, 3, 2, 2, 1, 1, 3, 7, labels=np.array([[-1, 0, 0, 1]] * 3), direct=True)


def test_benchmark_useful_pairs_from_the_oracle():
    """The useful-FLOP count bench.py reports for config 2 (unmasked pairs of
    the block plan, counted on the GPU: 209 222 076) equals the oracle's
    unit-scale count of the reference mask."""
    import torch

    from multics_b200.synth import CONFIGS, group_labels

    cfg = CONFIGS["cfg2"]  # static groups: labels do not depend on the generator
    lab = group_labels(cfg, torch.Generator().manual_seed(cfg.seed)).numpy()
    pairs = O.logical_pairs_units(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG, cfg.n_block,
                                  cfg.local_attn, labels=lab, direct=cfg.direct)
    assert pairs == 209222076


@pytest.mark.parametrize("case", [
    dict(P=4, T=3, L=5, N=2, KL=3, KG=2, n=1, win=-1, labels=[[0, 0, 1, 1]] * 3),
    dict(P=3, T=6, L=4, N=3, KL=2, KG=3, n=2, win=3, labels=[[0, 1, 1], [0, 1, 1], [2, 2, 0],
                                                              [2, 2, 0], [1, 0, 0], [1, 0, 0]]),
    dict(P=3, T=4, L=3, N=2, KL=4, KG=0, n=1, win=-1, labels=[[0, 0, 0]] * 4),
])
def test_unit_scale_pair_count_equals_dense_popcount(case):
    """Unit-scale count (with the inactive-hub self edge as a diagonal) equals
    the token-level popcount, labels and membership groupings."""
    c = dict(case)
    lab = np.array(c.pop("labels"))
    dims = (c["P"], c["T"], c["L"], c["N"], c["KL"], c["KG"], c["n"], c["win"])
    assert O.logical_pairs_units(*dims, labels=lab, direct=True) == \
        O.logical_pairs(*dims, labels=lab, direct=True)
    mem = np.zeros((c["T"], c["N"], c["P"]), bool)
    for t in range(c["T"]):
        for p in range(c["P"]):
            mem[t, lab[t, p], p] = True
    go = ~mem.any(1)
    go[:, 0] = True  # a global-only player
    assert O.logical_pairs_units(*dims, membership=mem, global_only=go, direct=True) == \
        O.logical_pairs(*dims, membership=mem, global_only=go, direct=True)

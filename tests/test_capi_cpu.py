"""CPU checks of the C-ABI library and of the host-side logic (no GPU calls)."""

import ctypes

import pytest
import torch

from multics_b200 import _lib


def test_library_loads_and_exports_every_declared_symbol():
    h = _lib.lib()
    declared = _lib.declared_symbols()
    assert declared, "no entry points parsed from include/hier_b200.h"
    for name in declared:
        assert hasattr(h, name), name
    assert set(_lib._SIGS) <= set(declared)
    assert h.hier_abi_version() >= 1


def test_error_path_reports_reference_exception_types():
    h = _lib.lib()
    # head_dim != 128 is refused before any device work
    rc = h.hier_attn_fwd(None, 0, 0, None, None, 0, 0, None, 0, 1, 64, None, 1, None, None, None,
                         1.0, None, None)
    assert rc == 2
    with pytest.raises(NotImplementedError, match="head_dim=128"):
        _lib.check(rc)
    g = _lib.HierGrouping()
    rc = h.hier_dense_mask(ctypes.byref(g), 0, 1, None, None)
    with pytest.raises(ValueError, match="invalid hierarchical dims"):
        _lib.check(rc)


def test_group_validation_messages_match_reference():
    from multics_b200.hier_masks import (_prepare_hier_group_tensors,
                                         _prepare_hier_membership_tensors,
                                         _refuse_membership_on_scalar_kernel,
                                         _slice_hier_active_group_for_cached_mask,
                                         make_grouping_spec)

    with pytest.raises(ValueError, match=r"must be in \[0,2\)"):
        _prepare_hier_group_tensors(torch.tensor([[-1, 0, 0, 1]] * 3), None, 4, 3, 2, "cpu")
    with pytest.raises(ValueError, match=r"group_labels must be \[T=3,P=4\]"):
        _prepare_hier_group_tensors(torch.zeros(2, 4, dtype=torch.long), None, 4, 3, 2, "cpu")
    lab, act = _prepare_hier_group_tensors(torch.tensor([[0, 0, 1, 1]] * 3), None, 4, 3, 3, "cpu")
    assert act.tolist() == [[True, True, False]] * 3
    with pytest.raises(ValueError, match="global_only"):
        _prepare_hier_membership_tensors(torch.zeros(3, 2, 4, dtype=torch.bool), None, None, 4, 3,
                                         2, "cpu")
    with pytest.raises(ValueError, match="does not cover cached block"):
        _slice_hier_active_group_for_cached_mask(torch.zeros(8, 2, dtype=torch.bool), 7, 2)
    with pytest.raises(ValueError, match="tiled128"):
        _refuse_membership_on_scalar_kernel(infer_kernel="tiled128")
    with pytest.raises(ValueError, match="hier_no_local_hub requires K_L=0"):
        make_grouping_spec(4, 3, 2, 2, 1, 1, 1, -1, torch.zeros(3, 4, dtype=torch.long),
                           hier_no_local_hub=True, device="cpu")
    with pytest.raises(NotImplementedError, match="CUDA"):
        make_grouping_spec(4, 3, 2, 2, 1, 1, 1, -1, torch.zeros(3, 4, dtype=torch.long),
                           device="cpu")


def test_shard_descriptor_validation_and_sizes():
    """hier_shard_sizes checks the shard descriptor on the host and sizes the
    plan: strips of the local players, hub-partial strips of its home
    players, hub-token pairs."""
    h = _lib.lib()

    def desc(players, strips, hp):
        d = _lib.HierShardDesc()
        d.P, d.N, d.L, d.KL, d.KG, d.T = 4, 2, 220, 16, 6, 42
        d.n_block, d.local_attn, d.direct = 1, -1, 1
        d.n_local, d.hub_keys = len(players), 1
        # grouping tables are device pointers, not read by the host checks
        d.labels = d.active = d.remote_key = 16
        for i, (p, (b, e), f) in enumerate(zip(players, strips, hp)):
            d.local_player[i], d.strip_begin[i], d.strip_end[i], d.hub_partials[i] = p, b, e, f
        return d

    sz = _lib.HierShardSizes()
    nps = -(-42 * 220 // 256)   # 37 strips of a player
    nph = -(-42 * 16 // 256)    # 3 hub-partial strips
    n_hh = 2 * nph + -(-42 * 6 // 256)
    d = desc([1, 2], [(20, nps), (0, 5)], [1, 0])
    _lib.check(h.hier_shard_sizes(ctypes.byref(d), ctypes.byref(sz)))
    assert sz.n_player_pairs == (nps - 20) + 5
    assert sz.n_pairs == sz.n_player_pairs + nph + n_hh
    assert sz.own_rows == 2 * 42 * 220 and sz.hub_partial_rows == 42 * 16
    assert sz.hub_rows == 42 * (2 * 16 + 6)
    for bad, msg in [(desc([], [], []), "holds 1..16 players"),
                     (desc([1, 1], [(0, 1), (1, 2)], [0, 0]), "listed twice"),
                     (desc([0], [(0, nps + 1)], [1]), "outside"),
                     (desc([7], [(0, 1)], [1]), "out of range")]:
        with pytest.raises(ValueError, match=msg):
            _lib.check(h.hier_shard_sizes(ctypes.byref(bad), ctypes.byref(sz)))


def test_sequence_plan_selection_rules(monkeypatch):
    """Which groupings the full-sequence entry points run on the sequence
    plan (labels, no no-local topology, T % n == 0, window -1 or >= n), and
    the environment switch to the block plan."""
    from types import SimpleNamespace

    from multics_b200.attention import FULL_SEQUENCE_PLAN_ENV, HierSequencePlan, sequence_plan

    base = dict(membership=None, labels=torch.zeros(6, 4, dtype=torch.long), no_local=False,
                T=6, n_block=3, local_attn=-1)
    ok = SimpleNamespace(**base)
    assert HierSequencePlan.supports(ok)
    for change in (dict(membership=torch.zeros(6, 2, 4, dtype=torch.bool)), dict(no_local=True),
                   dict(n_block=4), dict(local_attn=2), dict(labels=None)):
        assert not HierSequencePlan.supports(SimpleNamespace(**{**base, **change})), change
    assert HierSequencePlan.supports(SimpleNamespace(**{**base, "local_attn": 3}))
    mask = SimpleNamespace(spec=SimpleNamespace(**{**base, "no_local": True}))
    assert sequence_plan(mask, 2) is None  # unsupported grouping: block plan, no device work
    monkeypatch.setenv(FULL_SEQUENCE_PLAN_ENV, "blocks")
    assert sequence_plan(SimpleNamespace(spec=ok), 2) is None
    monkeypatch.setenv(FULL_SEQUENCE_PLAN_ENV, "tiles")
    with pytest.raises(ValueError, match="segments"):
        sequence_plan(SimpleNamespace(spec=ok), 2)


def test_plan_check_rejects_bad_arguments_on_the_host():
    """hier_plan_check refuses invalid sizes (no streams, more than 32, a
    negative count, missing tables) before any device work."""
    import ctypes

    from multics_b200 import _lib

    h = _lib.lib()
    rows1 = (ctypes.c_int64 * 1)(100)
    rows33 = (ctypes.c_int64 * 33)(*([100] * 33))
    st = ctypes.c_void_p(16)  # never written: the host check fails first
    for args in [(None, 0, None, 0, 0, None, 100, rows1, 0, st, None),
                 (None, 0, None, 0, 0, None, 100, rows33, 33, st, None),
                 (None, -1, None, 0, 0, None, 100, rows1, 1, st, None),
                 (None, 4, None, 0, 0, None, 100, rows1, 1, st, None),
                 (None, 0, None, 0, 0, None, 100, None, 1, st, None),
                 (None, 0, None, 0, 0, None, 100, rows1, 1, None, None)]:
        assert h.hier_plan_check(*args) == 1, args
        assert b"hier_plan_check" in h.hier_last_error()


def test_hub_lse_merges_partials_on_cpu():
    """HierSequencePlan.hub_lse: a hub row's log2-sum-exp is log2 of the sum
    of 2^lse over its partial rows (ragged lists, -inf partials, a row
    without keys), written at the row's sequence position."""
    from types import SimpleNamespace

    import numpy as np

    from multics_b200.attention import HierSequencePlan

    H = 3
    rng = np.random.default_rng(0)
    part = rng.normal(0, 4, (9, H)).astype(np.float32)
    part[2, 1] = -np.inf
    off = np.array([0, 3, 4, 7, 9], np.int32)
    rows = np.array([8, 7, 6, 5, 4, 3, 2, 1, 0], np.int32)
    part[[1, 0]] = -np.inf                    # target 3's partials: no keys at all
    dst = np.array([10, 12, 11, 13], np.int32)
    core = SimpleNamespace(csr_off=torch.from_numpy(off), csr_rows=torch.from_numpy(rows),
                           part_lse=torch.from_numpy(part))
    sp = SimpleNamespace(core=core, hub_dst=torch.from_numpy(dst))
    lse = torch.full((14, H), 7.0)
    HierSequencePlan.hub_lse(sp, lse)
    for t in range(4):
        vals = part[rows[off[t]:off[t + 1]]].astype(np.float64)
        with np.errstate(divide="ignore"):
            want = np.log2(np.exp2(vals).sum(0))
        np.testing.assert_allclose(lse[dst[t]].numpy(), want, rtol=1e-5, atol=1e-5)
    assert bool((lse[:10] == 7.0).all())      # other rows untouched
    assert bool(torch.isinf(lse[13]).all())

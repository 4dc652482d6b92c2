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

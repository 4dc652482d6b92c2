"""GPU check of the allocation-free block-mask entry point.

``hier_block_mask_build_static`` is for callers that cannot allocate device
memory while they run - a serving loop whose device memory is fully
pre-reserved by its own allocator, or a foreign-language binding with no
device allocator to provide a workspace.  It keeps its scratch in a fixed
device array inside the library instead of a caller workspace.  This test
calls it through the C ABI twice in a row, on two different groupings, and
checks that its outputs equal those of the workspace entry point
``hier_block_mask_build`` exactly (the outputs are integer block lists).  The
file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from helpers import mask_case

pytestmark = pytest.mark.gpu


def _spec(name, dev):
    from multics_b200.hier_masks import make_grouping_spec

    c = mask_case(name)
    t = lambda a, dt: None if a is None else torch.as_tensor(np.asarray(a), dtype=dt, device=dev)  # noqa: E731
    return make_grouping_spec(
        c["P"], c["T"], c["L"], c["N"], c["KL"], c["KG"], c["n"], c["win"],
        t(c["labels"], torch.long), t(c["active"], torch.bool), c["direct"], dev,
        t(c["membership"], torch.bool), t(c["global_only"], torch.bool), c["no_local"])


def _outputs(nb, dev):
    i32 = dict(dtype=torch.int32, device=dev)
    # poison the outputs so that unwritten entries cannot match by accident
    return {"kv_num": torch.full((nb,), -7, **i32), "kv_off": torch.full((nb + 1,), -7, **i32),
            "kv_idx": torch.full((nb * nb,), -7, **i32), "full_num": torch.full((nb,), -7, **i32),
            "full_off": torch.full((nb + 1,), -7, **i32),
            "full_idx": torch.full((nb * nb,), -7, **i32), "totals": torch.full((2,), -7, **i32)}


ORDER = ("kv_num", "kv_off", "kv_idx", "full_num", "full_off", "full_idx", "totals")


def _run_workspace(spec, dev):
    from multics_b200 import _lib
    from multics_b200._lib import check, ptr, stream_ptr

    L = _lib.lib()
    g = spec.c_struct()
    nb = (spec.S + 127) // 128
    ws_bytes = ctypes.c_size_t()
    check(L.hier_block_workspace_size(ctypes.byref(g), ctypes.byref(ws_bytes)))
    ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device=dev)
    out = _outputs(nb, dev)
    check(L.hier_block_mask_build(ctypes.byref(g), ptr(ws), *(ptr(out[k]) for k in ORDER),
                                  stream_ptr()))
    return out


def _run_static(spec, dev):
    from multics_b200 import _lib
    from multics_b200._lib import check, ptr, stream_ptr

    g = spec.c_struct()
    nb = (spec.S + 127) // 128
    out = _outputs(nb, dev)
    check(_lib.lib().hier_block_mask_build_static(ctypes.byref(g), *(ptr(out[k]) for k in ORDER),
                                                  stream_ptr()))
    return out


def _compare(a, b):
    torch.cuda.synchronize()
    n_partial, n_full = (int(x) for x in a["totals"].tolist())
    assert a["totals"].tolist() == b["totals"].tolist()
    for key in ("kv_num", "kv_off", "full_num", "full_off"):
        assert torch.equal(a[key], b[key]), key
    assert torch.equal(a["kv_idx"][:n_partial], b["kv_idx"][:n_partial])
    assert torch.equal(a["full_idx"][:n_full], b["full_idx"][:n_full])


def test_static_scratch_block_mask_matches_workspace_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    # two calls in a row on different groupings (the second finds the first's
    # contents in the shared scratch), then the first grouping again
    for name in ("fixture_p10_moving_pairs", "dyn_p8", "fixture_p10_moving_pairs"):
        spec = _spec(name, dev)
        _compare(_run_workspace(spec, dev), _run_static(spec, dev))


def test_static_scratch_rejects_oversized_problems():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from multics_b200 import _lib
    from multics_b200.hier_masks import make_grouping_spec

    dev = torch.device("cuda", 0)
    # 40 players x 42 frames x 220 tokens: ~2900 key blocks, ~8.5 MB of scratch
    spec = make_grouping_spec(40, 42, 220, 20, 16, 6, 1, -1,
                              (torch.arange(40, device=dev) // 2).repeat(42, 1), None, True, dev)
    g = spec.c_struct()
    rc = _lib.lib().hier_block_mask_build_static(ctypes.byref(g), *([None] * 7), None)
    with pytest.raises(ValueError, match="fixed .*-byte buffer"):
        _lib.check(rc)

"""Failure detection on the GPU without a GPU fault: the bounded pipeline
wait, given a short limit and a barrier phase that nothing completes, gives
up, reports DEV_WAIT_TIMEOUT with its wait site through the device error
word, and leaves the context usable.  Every wait of the library's kernels
goes through the same routine (with a limit of about two seconds)."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV_WAIT_TIMEOUT = 1
SITE = 30


def test_wait_gives_up_and_reports():
    from multics_b200 import _lib
    from multics_b200._lib import ptr, stream_ptr

    dev = torch.device("cuda")
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    cycles = torch.zeros(1, dtype=torch.int64, device=dev)
    limit = 2_000_000  # about a millisecond of SM clock
    t0 = time.perf_counter()
    _lib.check(_lib.lib().hier_selftest_wait_timeout(limit, ptr(err), ptr(cycles), stream_ptr()))
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    assert int(err.item()) == DEV_WAIT_TIMEOUT | (SITE << 8)
    assert limit <= int(cycles.item()) < 50 * limit
    assert wall < 2.0
    # the context still works, and an error word already set is kept
    x = torch.arange(1 << 20, device=dev, dtype=torch.float32)
    assert float(x.sum()) == float((1 << 20) * ((1 << 20) - 1) // 2)
    err2 = torch.full((1,), 7, dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().hier_selftest_wait_timeout(limit, ptr(err2), ptr(cycles), stream_ptr()))
    torch.cuda.synchronize()
    assert int(err2.item()) == 7


def test_wait_limit_is_checked():
    from multics_b200 import _lib
    from multics_b200._lib import ptr, stream_ptr

    dev = torch.device("cuda")
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    cycles = torch.zeros(1, dtype=torch.int64, device=dev)
    with pytest.raises(ValueError, match="wait limit"):
        _lib.check(_lib.lib().hier_selftest_wait_timeout(0, ptr(err), ptr(cycles), stream_ptr()))
    with pytest.raises(ValueError, match="wait limit"):
        _lib.check(_lib.lib().hier_selftest_wait_timeout(10**12, ptr(err), ptr(cycles),
                                                         stream_ptr()))

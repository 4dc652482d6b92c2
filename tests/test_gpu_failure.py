"""Failure detection on the GPU without a GPU fault: the bounded pipeline
wait, given a short limit and a barrier phase that nothing completes, gives
up, reports DEV_WAIT_TIMEOUT with its wait site through the device error
word, and leaves the context usable.  Every wait of the library's kernels
goes through the same routine (with a limit of about two seconds).

A corrupted work plan is rejected before any launch: ``hier_plan_check``
reports each kind of out-of-range index (only the check runs on the
corrupted copies), and ``MULTICS_B200_CHECK_PLANS=1`` runs it ahead of the
attention launch on a valid plan without changing the result."""

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


def _plan_case():
    from multics_b200.attention import attention_mask_plan

    dev = torch.device("cuda")
    S = 300
    g = torch.Generator(device="cuda").manual_seed(3)
    m = torch.rand(S, S, generator=g, device=dev) < 0.35
    m[:, 0] = True
    return attention_mask_plan(m, S, dev), S


def test_corrupted_plans_are_rejected_before_launch():
    from types import SimpleNamespace

    from multics_b200.attention import check_plan

    bm, S = _plan_case()
    check_plan(bm, S, S)
    qp0 = bm.q_pairs.cpu()
    e0 = int(qp0[0, 4])
    assert int(qp0[0, 5]) > e0 and int(qp0[0, 1]) > 0
    n_pairs, n_tiles = bm.q_pairs.shape[0], bm.kv_tiles.shape[0]
    n_masks = bm.row_masks.shape[0]
    cases = [("q_pairs", (0, 5), n_tiles + 3, "key-tile range"),
             ("q_pairs", (0, 4), -1, "key-tile range"),
             ("q_pairs", (0, 0), S + 200, "query rows"),
             ("kv_tiles", (e0, 2), n_masks + 7, "mask selector"),
             ("kv_tiles", (e0, 3), -3, "mask selector"),
             ("kv_tiles", (e0, 0), 5 << 24, "key box"),
             ("kv_tiles", (e0, 1), S + 64, "key box")]
    if bm.order is not None:
        cases.append(("order", (0,), n_pairs + 1, "order entry"))
    for field, idx, value, msg in cases:
        plan = SimpleNamespace(q_pairs=bm.q_pairs.clone(), kv_tiles=bm.kv_tiles.clone(),
                               row_masks=bm.row_masks,
                               order=None if bm.order is None else bm.order.clone())
        getattr(plan, field)[idx] = value
        with pytest.raises(ValueError, match=msg):
            check_plan(plan, S, S)


def test_plan_check_before_launch_keeps_the_result(monkeypatch):
    from multics_b200.attention import PLAN_CHECK_ENV, attention_from_plan, device_error

    bm, S = _plan_case()
    H = 2
    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, v = (torch.randn(S, H * 128, generator=g, device="cuda").bfloat16() for _ in range(3))
    ref = attention_from_plan(q, k, v, bm, H)
    monkeypatch.setenv(PLAN_CHECK_ENV, "1")
    got = attention_from_plan(q, k, v, bm, H)
    torch.cuda.synchronize()
    assert device_error() == 0
    assert torch.equal(got, ref)


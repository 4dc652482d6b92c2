"""Rolling-cache bookkeeping on CPU tensors: append, windowed eviction, and
refresh of an already-seen block (the reference's rules,
multics/models/attention.py:90-228)."""

import torch

from multics_b200.kv_cache import (new_stream_cache, rolling_bool_cache_append,
                                   rolling_cache_append)


def _vals(lo, hi):
    t = torch.arange(lo, hi, dtype=torch.float32)
    return t.view(1, -1, 1, 1)


def test_append_evict_refresh():
    c = new_stream_cache(1, 4, 1, 1, torch.float32, "cpu", with_active=True)
    # blocks of 2 tokens (1 token per frame), window 2 frames -> retention 4
    for blk in range(3):
        lo, hi = 2 * blk, 2 * blk + 2
        rolling_bool_cache_append(c, "active", torch.tensor([True, blk != 1]), lo, hi, 2, 0, 1)
        out = rolling_cache_append(c, _vals(lo, hi), -_vals(lo, hi), lo, hi, 2, 0, 1)
    assert int(c["global_end_index"]) == 6 and int(c["local_end_index"]) == 4
    assert c["k"].flatten().tolist() == [2, 3, 4, 5]
    assert c["v"].flatten().tolist() == [-2, -3, -4, -5]
    assert c["active"].tolist() == [True, False, True, True]
    assert out == (2, 4)  # attended window: the last 2 frames
    # the same block again (e.g. another denoising step) refreshes in place
    rolling_bool_cache_append(c, "active", torch.tensor([False, False]), 4, 6, 2, 0, 1)
    rolling_cache_append(c, 10 + _vals(4, 6), _vals(4, 6), 4, 6, 2, 0, 1)
    assert c["k"].flatten().tolist() == [2, 3, 14, 15]
    assert c["active"].tolist() == [True, False, False, False]
    assert int(c["global_end_index"]) == 6 and int(c["local_end_index"]) == 4


def test_unbounded_window_keeps_every_token():
    c = new_stream_cache(1, 9, 1, 1, torch.float32, "cpu")
    for blk in range(3):
        out = rolling_cache_append(c, _vals(3 * blk, 3 * blk + 3), _vals(0, 3), 3 * blk,
                                   3 * blk + 3, -1, 0, 3)
    assert int(c["local_end_index"]) == 9 and out == (0, 9)
    assert c["k"].flatten().tolist() == list(range(9))

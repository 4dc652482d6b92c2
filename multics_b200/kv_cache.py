"""Rolling key/value caches of the cached hierarchical forward.

Same dict format and update rules as the reference's
``_rolling_cache_append`` / ``_rolling_bool_cache_append``
(``multics/models/attention.py:90-228``), so a cache filled here is
interchangeable with one filled by the reference:

* a stream cache is ``{"k", "v": [B, capacity, H, D], "global_end_index",
  "local_end_index": long [1]}`` (+ ``"active": bool [capacity]`` for local
  hubs); ``global_end_index`` counts every token ever appended,
  ``local_end_index`` the tokens held;
* appending a block ``[current_start, current_end)`` writes the tokens past
  ``global_end_index`` (or refreshes the overlap when the block was seen
  before), evicting the oldest tokens (beyond ``sink`` frames) when a windowed
  cache overflows.

The caches live on the GPU; the two indices are read once per append, as in
the reference.
"""

from __future__ import annotations

import torch

__all__ = ["new_stream_cache", "new_hier_cache", "rolling_cache_append",
           "rolling_bool_cache_append"]


def new_stream_cache(batch, capacity, heads, head_dim, dtype, device, with_active=False):
    c = {"k": torch.zeros(batch, capacity, heads, head_dim, dtype=dtype, device=device),
         "v": torch.zeros(batch, capacity, heads, head_dim, dtype=dtype, device=device),
         "global_end_index": torch.zeros(1, dtype=torch.long, device=device),
         "local_end_index": torch.zeros(1, dtype=torch.long, device=device)}
    if with_active:
        c["active"] = torch.zeros(capacity, dtype=torch.bool, device=device)
    return c


def new_hier_cache(*, num_players, num_groups, num_local_hub_tokens, num_global_hub_tokens,
                   frame_seq_length, retention_frames, heads, head_dim, dtype, device,
                   no_local=False, batch=1):
    """One layer's cache in the format the pipeline builds
    (``multics/pipelines/wan_video_Nplayers.py:888-979``)."""
    P, N, KL, KG, L = (num_players, num_groups, num_local_hub_tokens, num_global_hub_tokens,
                       frame_seq_length)
    r = retention_frames
    return {
        "sparse_hub": True, "hier_hub": True, "num_players": P, "num_hub_tokens": N * KL + KG,
        "num_groups": N, "num_local_hub_tokens": KL, "num_global_hub_tokens": KG,
        "hier_no_local_hub": bool(no_local), "frame_seq_length": L,
        "agent_caches": [new_stream_cache(batch, r * L, heads, head_dim, dtype, device)
                         for _ in range(P)],
        "local_hubs": [] if no_local else [
            new_stream_cache(batch, r * max(KL, 1), heads, head_dim, dtype, device, True)
            for _ in range(N)],
        "global_hub": new_stream_cache(batch, r * max(KG, 1), heads, head_dim, dtype, device),
    }


def _window_update(capacity, current_global_end, current_local_end, n_in, current_start,
                   current_end, local_attn_size, sink_tokens):
    """Index arithmetic shared by both appends: returns (refresh, roll,
    new_local_end, num_new) where refresh = (src, dst, len) or None and roll =
    (src, dst, len) or None."""
    progress = max(0, current_end - current_global_end)
    num_new = min(n_in, progress)
    refresh = None
    if num_new == 0 and current_local_end > 0:
        cached_start = current_global_end - current_local_end
        r0 = max(current_start, cached_start)
        r1 = min(current_end, current_global_end)
        if r1 > r0:
            refresh = (r0 - current_start, r0 - cached_start, r1 - r0)
    new_local_end = current_local_end + num_new
    roll = None
    if local_attn_size != -1 and current_end > current_global_end and new_local_end > capacity:
        evict = max(0, min(new_local_end - capacity, new_local_end - sink_tokens - 1))
        if evict > 0:
            rolled = max(0, current_local_end - evict - sink_tokens)
            if rolled > 0:
                roll = (sink_tokens + evict, sink_tokens, rolled)
            new_local_end = min(current_local_end + num_new - evict, capacity)
    return refresh, roll, new_local_end, num_new


def rolling_cache_append(kv_cache, roped_key, value, current_start, current_end,
                         local_attn_size, sink_size, tokens_per_frame):
    """Append or refresh keys/values of a block in a rolling cache; returns
    ``(attn_start, local_end)`` of the attended window."""
    sink_tokens = sink_size * tokens_per_frame
    capacity = kv_cache["k"].shape[1]
    g_end = int(kv_cache["global_end_index"].item())
    l_end = int(kv_cache["local_end_index"].item())
    refresh, roll, new_end, num_new = _window_update(
        capacity, g_end, l_end, roped_key.shape[1], current_start, current_end,
        local_attn_size, sink_tokens)
    k, v = kv_cache["k"], kv_cache["v"]
    if refresh is not None:
        src, dst, n = refresh
        k[:, dst:dst + n] = roped_key[:, src:src + n]
        v[:, dst:dst + n] = value[:, src:src + n]
    if roll is not None:
        src, dst, n = roll
        k[:, dst:dst + n] = k[:, src:src + n].clone()
        v[:, dst:dst + n] = v[:, src:src + n].clone()
    if num_new > 0:
        s0 = new_end - num_new
        k[:, s0:s0 + num_new] = roped_key[:, -num_new:]
        v[:, s0:s0 + num_new] = value[:, -num_new:]
    max_attn = capacity if local_attn_size == -1 else min(local_attn_size * tokens_per_frame,
                                                          capacity)
    attn_start = max(0, new_end - max_attn)
    if sink_size > 0 and sink_tokens > attn_start:
        attn_start = 0
    kv_cache["global_end_index"].fill_(current_end)
    kv_cache["local_end_index"].fill_(new_end)
    return attn_start, new_end


def rolling_bool_cache_append(kv_cache, key, values, current_start, current_end,
                              local_attn_size, sink_size, tokens_per_frame):
    """Append/refresh a 1-D bool side cache in lockstep with the K/V cache
    (called before :func:`rolling_cache_append`, which moves the indices)."""
    if key not in kv_cache:
        return
    sink_tokens = sink_size * tokens_per_frame
    cache = kv_cache[key]
    g_end = int(kv_cache["global_end_index"].item())
    l_end = int(kv_cache["local_end_index"].item())
    refresh, roll, new_end, num_new = _window_update(
        cache.shape[0], g_end, l_end, values.shape[0], current_start, current_end,
        local_attn_size, sink_tokens)
    if refresh is not None:
        src, dst, n = refresh
        cache[dst:dst + n] = values[src:src + n]
    if roll is not None:
        src, dst, n = roll
        cache[dst:dst + n] = cache[src:src + n].clone()
    if num_new > 0:
        s0 = new_end - num_new
        cache[s0:s0 + num_new] = values[-num_new:]

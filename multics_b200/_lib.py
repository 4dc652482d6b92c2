"""ctypes binding of libhier_b200.so (the C ABI declared in include/hier_b200.h).

The library is required: there is no CPU or PyTorch fallback for any entry
point.  Loading fails loudly with the build command if the in-tree library is
missing.
"""

from __future__ import annotations

import ctypes
import re
from ctypes import c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libhier_b200.so"
HEADER = PKG.parent / "include" / "hier_b200.h"

HIER_OK = 0
_EXC = {1: ValueError, 2: NotImplementedError, 3: RuntimeError, 4: AssertionError, 5: RuntimeError}


class HierGrouping(ctypes.Structure):
    """Mirror of ``struct hier_grouping`` in include/hier_b200.h."""

    _fields_ = [
        ("P", c_int32), ("T", c_int32), ("L", c_int32), ("N", c_int32), ("KL", c_int32),
        ("KG", c_int32), ("n_block", c_int32), ("local_attn", c_int32), ("direct", c_int32),
        ("no_local", c_int32), ("membership_mode", c_int32), ("labels", c_void_p),
        ("membership", c_void_p), ("global_only", c_void_p), ("active", c_void_p),
    ]


MAX_KV_STREAMS = 32
SHARD_MAX_LOCAL = 16


class HierCachedGrouping(ctypes.Structure):
    """Mirror of ``struct hier_cached_grouping`` in include/hier_b200.h."""

    _fields_ = [
        ("P", c_int32), ("N", c_int32), ("L", c_int32), ("KL", c_int32), ("KG", c_int32),
        ("n_frames", c_int32), ("n_block", c_int32), ("local_attn", c_int32),
        ("direct", c_int32), ("no_local", c_int32), ("membership_mode", c_int32),
        ("fa", c_int32), ("fl", c_int32), ("fg", c_int32), ("T_mem", c_int32),
        ("agent_frames", c_void_p * MAX_KV_STREAMS),
        ("local_frames", c_void_p * MAX_KV_STREAMS),
        ("local_active", c_void_p * MAX_KV_STREAMS),
        ("global_frames", c_void_p), ("labels", c_void_p), ("q_active", c_void_p),
        ("membership", c_void_p), ("global_only", c_void_p),
    ]


class HierCachedPackSizes(ctypes.Structure):
    """Mirror of ``hier_cached_pack_sizes_t``."""

    _fields_ = [("n_packs", ctypes.c_int32), ("q2_rows", ctypes.c_int32),
                ("agent_pairs", ctypes.c_int32), ("tile_capacity", ctypes.c_int32)]


class HierCachedSizes(ctypes.Structure):
    """Mirror of ``hier_cached_sizes_t``."""

    _fields_ = [
        ("n_seg", c_int32), ("n_prog", c_int32), ("n_pairs", c_int32), ("n_streams", c_int32),
        ("n_cand", c_int32), ("tile_capacity", c_int32), ("q_rows", c_int64),
        ("pool_rows", c_int64),
    ]


class HierTiledGrouping(ctypes.Structure):
    """Mirror of ``struct hier_tiled_grouping``."""

    _fields_ = [
        ("mode", c_int32), ("P", c_int32), ("N", c_int32), ("L", c_int32), ("KL", c_int32),
        ("KG", c_int32), ("n_block", c_int32), ("local_attn", c_int32), ("direct", c_int32),
        ("T", c_int32), ("n_frames", c_int32), ("fa", c_int32), ("fl", c_int32), ("fg", c_int32),
        ("labels", c_void_p), ("active", c_void_p),
        ("agent_frames", c_void_p * MAX_KV_STREAMS),
        ("local_frames", c_void_p * MAX_KV_STREAMS),
        ("local_active", c_void_p * MAX_KV_STREAMS),
        ("global_frames", c_void_p),
    ]


class HierTiledSizes(ctypes.Structure):
    """Mirror of ``hier_tiled_sizes_t``."""

    _fields_ = [
        ("n_layouts", c_int32), ("n_seg", c_int32), ("n_prog", c_int32), ("n_pairs", c_int32),
        ("tile_capacity", c_int32), ("reserved", c_int32), ("q_rows", c_int64),
    ]


class HierShardDesc(ctypes.Structure):
    """Mirror of ``struct hier_shard_desc``."""

    _fields_ = [
        ("P", c_int32), ("N", c_int32), ("L", c_int32), ("KL", c_int32), ("KG", c_int32),
        ("T", c_int32), ("n_block", c_int32), ("local_attn", c_int32), ("direct", c_int32),
        ("n_local", c_int32), ("hub_keys", c_int32), ("hub_partial_row0", c_int32),
        ("labels", c_void_p), ("active", c_void_p), ("remote_key", c_void_p),
        ("local_player", c_int32 * SHARD_MAX_LOCAL), ("strip_begin", c_int32 * SHARD_MAX_LOCAL),
        ("strip_end", c_int32 * SHARD_MAX_LOCAL), ("hub_partials", c_int32 * SHARD_MAX_LOCAL),
        ("page_table", c_void_p), ("n_pages", c_int32), ("hub_key_first", c_int32),
        ("hub_key_count", c_int32),
    ]


class HierShardSizes(ctypes.Structure):
    """Mirror of ``hier_shard_sizes_t``."""

    _fields_ = [
        ("n_pairs", c_int32), ("n_player_pairs", c_int32), ("n_counts", c_int32),
        ("reserved", c_int32), ("own_rows", c_int64), ("hub_rows", c_int64),
        ("hub_partial_rows", c_int64),
    ]


class HierPartialOut(ctypes.Structure):
    """Mirror of ``hier_partial_out``."""

    _fields_ = [
        ("q2", c_void_p), ("q2_rows", c_int64), ("q2_stride", c_int64), ("q2_row0", c_int64),
        ("o", c_void_p), ("o_stride", c_int64), ("lse", c_void_p), ("row0", c_int64),
        ("slot_rows", c_int64),
    ]


_P = c_void_p
_SIGS = {
    "hier_last_error": (c_char_p, []),
    "hier_last_error_code": (c_int, []),
    "hier_abi_version": (c_int, []),
    "hier_dense_mask": (c_int, [ctypes.POINTER(HierGrouping), c_int64, c_int64, _P, _P]),
    "hier_block_workspace_size": (c_int, [ctypes.POINTER(HierGrouping), ctypes.POINTER(c_size_t)]),
    "hier_block_mask_build": (c_int, [ctypes.POINTER(HierGrouping), _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "hier_block_plan_build": (c_int, [ctypes.POINTER(HierGrouping), _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                      _P, _P, _P]),
    "hier_block_mask_build_static": (c_int, [ctypes.POINTER(HierGrouping), _P, _P, _P, _P, _P, _P, _P,
                                             _P]),
    "hier_dense_block_workspace_size": (c_int, [c_int64, ctypes.POINTER(c_size_t)]),
    "hier_dense_block_mask_build": (c_int, [_P, c_int64, c_int64, _P, _P, _P, _P, _P, _P, _P, _P,
                                            _P]),
    "hier_dense_block_plan_build": (c_int, [_P, c_int64, c_int64, _P, _P, _P, _P, _P, _P, _P, _P,
                                            _P]),
    "hier_plan_split_kv": (c_int, [_P, c_int32, c_int32, _P, _P, _P]),
    "hier_shared_mask_plan_size": (c_int, [c_int64, c_int64, c_int64, c_int32, _P, _P]),
    "hier_prep_qk_bwd_partials": (c_int, [c_int64, _P]),
    "hier_prep_qk_bwd": (c_int, [_P, _P, c_int64, _P, c_int32, _P, _P, _P, _P, _P, c_int64,
                                 c_int64, c_int32, c_int32, c_float, _P, _P, c_int64, _P, _P,
                                 c_int64, _P, _P]),
    "hier_attn_bwd_prep": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, c_int32, c_int32, _P,
                                   _P, c_int64, _P]),
    "hier_bwd_plan_transpose": (c_int, [_P, c_int32, _P, _P, c_int32, c_int32, _P, _P, _P,
                                        c_int32, _P, _P, _P]),
    "hier_attn_bwd_dq": (c_int, [_P, c_int64, c_int64, _P, _P, c_int64, c_int64, _P, c_int64, _P,
                                 _P, c_int64, c_int32, c_int32, _P, c_int32, _P, _P, c_int32,
                                 c_float, _P, c_int64, _P, _P]),
    "hier_attn_bwd_dkv": (c_int, [_P, c_int64, c_int64, _P, _P, c_int64, c_int64, _P, c_int64, _P,
                                  _P, c_int64, c_int32, c_int32, _P, _P, _P, c_int32, c_float, _P,
                                  c_int64, _P, c_int64, _P, _P]),
    "hier_shared_mask_plan_build": (c_int, [_P, c_int64, c_int64, c_int64, c_int64, c_int32, _P,
                                            _P, _P, _P, _P]),
    "hier_prep_qk": (c_int, [_P, _P, c_int64, _P, c_int32, _P, _P, _P, _P, _P, c_int64, c_int64,
                             c_int32,
                             c_int32, c_float, _P, _P, c_int64, _P, _P, _P]),
    "hier_attn_fwd": (c_int, [_P, c_int64, c_int64, _P, _P, c_int64, c_int64, _P, c_int64, c_int32,
                              c_int32, _P, c_int32, _P, _P, _P, c_float, _P, _P]),
    "hier_attn_fwd_streams": (c_int, [_P, c_int64, c_int64, c_int32, _P, _P, _P, _P, _P, c_int64,
                                      _P, c_int32, c_int32, _P, c_int32, _P, _P, c_int32, _P,
                                      c_float, _P, ctypes.POINTER(HierPartialOut), _P, _P]),
    "hier_cached_sizes": (c_int, [ctypes.POINTER(HierCachedGrouping), c_int32,
                                  ctypes.POINTER(HierCachedSizes)]),
    "hier_cached_count": (c_int, [ctypes.POINTER(HierCachedGrouping), _P, _P, _P, _P]),
    "hier_cached_pack_sizes": (c_int, [ctypes.POINTER(HierCachedGrouping),
                                       ctypes.POINTER(HierCachedPackSizes)]),
    "hier_cached_pack_count": (c_int, [ctypes.POINTER(HierCachedGrouping), _P, _P, _P]),
    "hier_cached_pack_build": (c_int, [ctypes.POINTER(HierCachedGrouping), _P, c_int32, c_int32,
                                       c_int32, c_int32, _P, _P, _P, _P, _P, _P]),
    "hier_cached_build": (c_int, [ctypes.POINTER(HierCachedGrouping), c_int32, _P, _P, _P, _P, _P,
                                  c_int32, _P, _P, _P, c_int32, _P, _P, _P]),
    "hier_varlen_workspace_size": (c_int, [c_int32, ctypes.POINTER(c_size_t)]),
    "hier_varlen_plan_build": (c_int, [_P, _P, _P, c_int32, _P, c_int32, _P, _P, _P, _P, _P, _P,
                                       _P, _P]),
    "hier_tiled_sizes": (c_int, [ctypes.POINTER(HierTiledGrouping), ctypes.POINTER(HierTiledSizes)]),
    "hier_tiled_count": (c_int, [ctypes.POINTER(HierTiledGrouping), _P, _P, _P, _P, _P]),
    "hier_tiled_build": (c_int, [ctypes.POINTER(HierTiledGrouping), _P, _P, _P, _P, _P, _P, _P, _P,
                                 _P, _P, _P, c_int32, _P, _P, _P]),
    "hier_shard_sizes": (c_int, [ctypes.POINTER(HierShardDesc), ctypes.POINTER(HierShardSizes)]),
    "hier_shard_count": (c_int, [ctypes.POINTER(HierShardDesc), _P, _P, _P, _P]),
    "hier_shard_build": (c_int, [ctypes.POINTER(HierShardDesc), _P, _P, _P, c_int32, _P, c_int64,
                                 _P, _P, _P]),
    "hier_lse_gather_merge": (c_int, [_P, c_int64, _P, c_int32, c_int32, _P, _P, c_int64, _P,
                                      c_int64, _P, _P]),
    "hier_lse_gather_merge_peers": (c_int, [_P, _P, c_int32, c_int32, c_int64, c_int64, c_int64,
                                            c_int32, c_int32, _P, _P, c_int64, _P, c_int64, _P,
                                            _P, _P]),
    "hier_plan_check": (c_int, [_P, c_int32, _P, c_int64, c_int64, _P, c_int64, _P, c_int32, _P,
                                _P]),
    "hier_selftest_umma": (c_int, [_P, _P, _P, _P, _P, _P, _P]),
    "hier_selftest_wait_timeout": (c_int, [c_int64, _P, _P, _P]),
}

_LIB = None

# hier_abi_version() of the library these signatures describe
ABI_VERSION = 5


def lib():
    """Load the in-tree library (once) and declare the C signatures."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m multics_b200.build` "
                "(the hierarchical attention path has no fallback implementation)")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        if h.hier_abi_version() != ABI_VERSION:
            raise RuntimeError(
                f"{LIB_PATH.name} has ABI version {h.hier_abi_version()}, the package expects "
                f"{ABI_VERSION}; rebuild it with `python -m multics_b200.build`")
        _LIB = h
    return _LIB


def declared_symbols():
    """Function names declared in include/hier_b200.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(hier_\w+)\s*\(", text, re.M)))


def check(rc: int):
    """Raise the reference's exception type for a non-zero status code."""
    if rc != HIER_OK:
        msg = lib().hier_last_error().decode(errors="replace")
        raise _EXC.get(rc, RuntimeError)(msg)


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else c_void_p(t.data_ptr())


def stream_ptr(device=None):
    import torch

    return c_void_p(torch.cuda.current_stream(device).cuda_stream)

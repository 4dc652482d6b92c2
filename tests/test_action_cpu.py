"""Action-branch attention on the CPU: the reference's masks and modules
pinned to the fixtures recorded from the reference itself
(``tests/golden/action.npz``), the mask helpers of ``multics_b200.action``
against them, and the host-side sizing of the shared-mask plan through the
C ABI (no GPU work)."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ref_cpu_path as R

GOLD = np.load(Path(__file__).parent / "golden" / "action.npz")


def _bf16(a):
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).float()


def _weights(prefix):
    w = {}
    for name in ("q", "k", "v", "o"):
        w[f"{name}.weight"] = _bf16(GOLD[f"{prefix}/{name}.weight"])
        w[f"{name}.bias"] = _bf16(GOLD[f"{prefix}/{name}.bias"])
    for name in ("norm_q", "norm_k"):
        w[f"{name}.weight"] = _bf16(GOLD[f"{prefix}/{name}.weight"])
    return w


@pytest.mark.parametrize("case", [tuple(c) for c in GOLD["mask_cases"]])
def test_temporal_masks_match_reference(case):
    from multics_b200.action import get_temporal_block_causal_mask

    F, n, win = (int(x) for x in case)
    gold = GOLD[f"temporal/{F}_{n}_{win}"]
    assert np.array_equal(R.temporal_block_causal_mask(F, n, win), gold)
    assert np.array_equal(get_temporal_block_causal_mask(F, n, win).numpy(), gold)


@pytest.mark.parametrize("case", [tuple(c) for c in GOLD["kb_cases"]])
def test_keyboard_masks_match_reference(case):
    from multics_b200.action import get_temporal_block_causal_mask, keyboard_frame_mask

    F, n, win, L = (int(x) for x in case)
    gold = GOLD[f"keyboard/{F}_{n}_{win}_{L}"]
    assert np.array_equal(R.keyboard_mask(R.temporal_block_causal_mask(F, n, win), L), gold)
    fm = get_temporal_block_causal_mask(F, n, win)
    assert np.array_equal(keyboard_frame_mask(fm, L).numpy(), gold)


def test_cached_frame_mask_is_the_frame_predicate():
    """The cached action attentions' mask over global frame indices equals
    the full temporal mask restricted to the query block and key window."""
    from multics_b200.action import cached_frame_mask

    F, n, win = 30, 3, 7
    full = R.temporal_block_causal_mask(F, n, win)
    gq = torch.arange(21, 24)
    gk = torch.arange(14, 24)
    m = cached_frame_mask(gq, gk, n, win).numpy()
    assert np.array_equal(m, full[21:24][:, 14:24])


def test_oracle_temporal_attention_matches_reference():
    B, F, n, win, H, D = (int(x) for x in GOLD["temporal/shape"])
    x = _bf16(GOLD["temporal/x"]).reshape(B, F, H * D)
    got = R.action_temporal_forward(x, _weights("temporal"), H,
                                    R.temporal_block_causal_mask(F, n, win))
    ref = torch.from_numpy(GOLD["temporal/out"])
    assert float((got - ref).abs().max()) < 1e-5


def test_oracle_keyboard_attention_matches_reference():
    P, F, n, win, L, K, H, D = (int(x) for x in GOLD["keyboard/shape"])
    x = _bf16(GOLD["keyboard/x"]).reshape(P, F * L, H * D)
    ctx = _bf16(GOLD["keyboard/ctx"]).reshape(P, F * K, H * D)
    mask = R.keyboard_mask(R.temporal_block_causal_mask(F, n, win), L, K)
    got = R.action_cross_forward(x, ctx, _weights("keyboard"), H, mask)
    ref = torch.from_numpy(GOLD["keyboard/out"])
    assert float((got - ref).abs().max()) < 1e-5


def _plan_size(B, Lq, Lk, aligned=0):
    from multics_b200 import _lib

    n, cap = ctypes.c_int32(), ctypes.c_int32()
    rc = _lib.lib().hier_shared_mask_plan_size(B, Lq, Lk, aligned, ctypes.byref(n),
                                               ctypes.byref(cap))
    return rc, n.value, cap.value


@pytest.mark.parametrize("B,Lq,Lk,pairs,cap", [
    (880, 42, 42, 147, 2),      # config 3 per-frame attention: 3 sequences per tile
    (4, 9240, 504, 146, 8),     # config 3 keyboard cross-attention: 73 tiles per player
    (1, 1, 1, 1, 2),
    (5, 64, 64, 2, 2),          # 2 per tile, 3 tiles
    (3, 128, 300, 2, 6),
    (2, 129, 7, 2, 2),          # a 129-row sequence: 2 tiles each
])
def test_shared_mask_plan_size(B, Lq, Lk, pairs, cap):
    rc, n, c = _plan_size(B, Lq, Lk)
    assert rc == 0 and (n, c) == (pairs, cap)


@pytest.mark.parametrize("B,Lq,Lk,pairs,cap", [
    (880, 42, 42, 145, 4),      # per-frame attention on the 128-row grid: 289 query tiles
    (4, 9240, 504, 145, 9),     # keyboard cross-attention: a pair spans 2 players' keys
    (1, 1, 1, 1, 1),
    (3, 128, 300, 2, 8),        # every key tile of the 900 rows
])
def test_aligned_shared_mask_plan_size(B, Lq, Lk, pairs, cap):
    rc, n, c = _plan_size(B, Lq, Lk, aligned=1)
    assert rc == 0 and (n, c) == (pairs, cap)


def test_shared_mask_plan_rejects_bad_sizes():
    from multics_b200 import _lib

    for B, Lq, Lk in ((0, 4, 4), (2, 0, 4), (2, 4, -1), (1 << 20, 8, 64)):
        rc, _, _ = _plan_size(B, Lq, Lk)
        assert rc == 1, (B, Lq, Lk)
        assert b"shared-mask plan" in _lib.lib().hier_last_error()


def test_out_refused_while_autograd_records():
    """The differentiable form allocates its own output: ``out=`` is refused
    (before any device work) when q, k or v requires grad."""
    import torch

    from multics_b200.action import shared_mask_attention

    q = torch.zeros(2, 4, 256, dtype=torch.bfloat16, requires_grad=True)
    k = torch.zeros(2, 6, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="out="):
        shared_mask_attention(q, k, k, 2, None, out=torch.empty_like(q))

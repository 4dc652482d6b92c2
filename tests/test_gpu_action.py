"""Action-branch attention on the GPU (the DiT block's per-frame mouse
attention and keyboard cross-attention, ``multics/models/blocks.py:677-697``).

* The shared-mask plan, packed and aligned, re-expands to exactly the
  batch's block-diagonal mask: every (query row, key row) pair is covered
  once, with the mask's bit; the aligned plan's tiles sit on the 128-row grid.
* ``shared_mask_attention`` matches an fp32 torch SDPA restatement
  (``oracle.ref_cpu_path.shared_mask_sdpa``) on random inputs, including
  rows without keys (0 here; SDPA gives NaN).
* ``SelfAttention`` over a batch and ``CrossAttention`` with the reference's
  weights reproduce the fp32 outputs recorded from the reference modules
  (``tests/golden/action.npz``).
* Configuration-3 sizes (880 sequences of 42 frames; 4 players x 9 240 query
  rows x 504 keyboard keys, 24 heads) against fp32 on sampled batches.
Tolerance as every attention test: max-abs <= 2e-2, cosine >= 0.9995.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ref_cpu_path as R

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995
GOLD = np.load(Path(__file__).parent / "golden" / "action.npz")


def _close(got, ref, what=""):
    got, ref = got.float(), ref.float()
    err = float((got - ref).abs().max())
    cos = float((got * ref).sum() / (got.norm() * ref.norm() + 1e-30))
    assert err <= MAX_ABS, (what, err)
    assert cos >= MIN_COS, (what, cos)


def _expand(plan, B, Lq, Lk):
    """Dense [B*Lq, B*Lk] coverage count and visibility of a plan."""
    qp = plan.q_pairs.cpu().numpy()
    kv = plan.kv_tiles.cpu().numpy()
    rm = plan.row_masks.cpu().numpy().view(np.uint32)
    cover = np.zeros((B * Lq, B * Lk + 256), np.int32)
    seen = np.zeros((B * Lq, B * Lk + 256), bool)
    row_cover = np.zeros(B * Lq, np.int32)
    bits = ((rm[:, :, :, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(rm.shape[0], 128, 128)
    for p in range(qp.shape[0]):
        halves = [(qp[p, 0], qp[p, 1]), (qp[p, 2], qp[p, 3])]
        for q0, nr in halves:
            row_cover[q0:q0 + nr] += 1
        for e in range(qp[p, 4], qp[p, 5]):
            k0, k1, m0, m1 = kv[e]
            assert k1 == k0 + 64
            keys = k0 + np.arange(128)
            for h, (q0, nr) in enumerate(halves):
                sel = (m0, m1)[h]
                if sel == -2 or nr == 0:
                    continue
                vis = np.ones((nr, 128), bool) if sel == -1 else bits[sel, :nr].astype(bool)
                cover[q0:q0 + nr, keys] += 1
                seen[q0:q0 + nr, keys] |= vis
    assert (row_cover == 1).all(), "every query row in exactly one tile"
    assert not seen[:, B * Lk:].any(), "no key beyond the last batch entry"
    return cover[:, :B * Lk], seen[:, :B * Lk]


PLAN_CASES = [
    (6, 42, 42, "temporal", (1, -1)),
    (7, 42, 42, "temporal", (7, 24)),
    (5, 64, 64, "temporal", (2, 3)),
    (3, 9 * 7, 9 * 12, "keyboard", (3, 4, 7)),
    (2, 30 * 11, 30 * 12, "keyboard", (2, -1, 11)),
    (3, 129, 200, "random", 0.3),
    (9, 5, 300, "random", 0.5),
    (4, 200, 17, "random", 0.1),
]


def _mask(kind, arg, Lq, Lk, seed=0):
    if kind == "temporal":
        return R.temporal_block_causal_mask(Lq, *arg)
    if kind == "keyboard":
        n, win, L = arg
        return R.keyboard_mask(R.temporal_block_causal_mask(Lq // L, n, win), L)
    rng = np.random.default_rng(seed)
    m = rng.random((Lq, Lk)) < arg
    m[1] = False  # a row without keys
    return m


@pytest.mark.parametrize("aligned", [False, True], ids=["packed", "aligned"])
@pytest.mark.parametrize("B,Lq,Lk,kind,arg", PLAN_CASES)
def test_shared_mask_plan_expands_to_block_diagonal(B, Lq, Lk, kind, arg, aligned):
    from multics_b200.action import SharedMaskPlan

    m = _mask(kind, arg, Lq, Lk)
    plan = SharedMaskPlan(torch.from_numpy(m).cuda(), B, aligned=aligned)
    torch.cuda.synchronize()
    if aligned:  # the form the backward's transpose takes
        qp, kv = plan.q_pairs.cpu(), plan.kv_tiles.cpu()
        assert bool((qp[:, [0, 2]] % 128 == 0).all())
        for p in range(qp.shape[0]):
            ks = kv[int(qp[p, 4]):int(qp[p, 5]), 0]
            assert bool((ks % 128 == 0).all()) and bool((ks[1:] > ks[:-1]).all())
    cover, seen = _expand(plan, B, Lq, Lk)
    want = np.kron(np.eye(B, dtype=bool), m)
    assert np.array_equal(seen, want)
    assert (cover[want] == 1).all(), "each visible pair exactly once"
    assert cover.max() <= 1


@pytest.mark.parametrize("B,Lq,Lk,kind,arg", PLAN_CASES)
def test_shared_mask_attention_matches_fp32(B, Lq, Lk, kind, arg):
    from multics_b200.action import shared_mask_attention
    from multics_b200.attention import device_error

    H = 2
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v = (torch.randn(B, L, H * 128, generator=g, device="cuda").bfloat16()
               for L in (Lq, Lk, Lk))
    m = torch.from_numpy(_mask(kind, arg, Lq, Lk)).cuda()
    err0 = device_error()
    out = shared_mask_attention(q, k, v, H, m)
    torch.cuda.synchronize()
    assert device_error() == err0 == 0
    ref = R.shared_mask_sdpa(q.float(), k.float(), v.float(), H, m)
    empty = ~m.any(1)
    if bool(empty.any()):
        assert bool((out[:, empty] == 0).all()), "rows without keys are 0"
        ref[:, empty] = 0
    _close(out, ref, (B, Lq, Lk, kind))


def test_shared_mask_attention_mask_forms():
    """[1, 1, Lq, Lk], a broadcast [1, Lk] mask, a uint8 mask and no mask."""
    from multics_b200.action import shared_mask_attention

    B, Lq, Lk, H = 3, 50, 70, 2
    g = torch.Generator(device="cuda").manual_seed(2)
    q, k, v = (torch.randn(B, L, H * 128, generator=g, device="cuda").bfloat16()
               for L in (Lq, Lk, Lk))
    m = torch.rand(Lq, Lk, generator=g, device="cuda") < 0.6
    m[:, 0] = True
    base = shared_mask_attention(q, k, v, H, m)
    assert torch.equal(shared_mask_attention(q, k, v, H, m[None, None]), base)
    assert torch.equal(shared_mask_attention(q, k, v, H, m.to(torch.uint8)), base)
    col = m[0:1]
    _close(shared_mask_attention(q, k, v, H, col),
           R.shared_mask_sdpa(q.float(), k.float(), v.float(), H, col.expand(Lq, Lk)), "row mask")
    _close(shared_mask_attention(q, k, v, H, None),
           R.shared_mask_sdpa(q.float(), k.float(), v.float(), H,
                              torch.ones(Lq, Lk, dtype=torch.bool, device="cuda")), "no mask")
    with pytest.raises(ValueError):
        shared_mask_attention(q, k, v, H, torch.ones(2, Lq, Lk, dtype=torch.bool, device="cuda"))


def _bf16(a):
    return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _load(module, prefix):
    with torch.no_grad():
        for name in ("q", "k", "v", "o"):
            getattr(module, name).weight.copy_(_bf16(GOLD[f"{prefix}/{name}.weight"]))
            getattr(module, name).bias.copy_(_bf16(GOLD[f"{prefix}/{name}.bias"]))
        for name in ("norm_q", "norm_k"):
            getattr(module, name).weight.copy_(_bf16(GOLD[f"{prefix}/{name}.weight"]))
    return module


def test_temporal_self_attention_matches_reference_module():
    """``SelfAttention`` over a batch of frame sequences with the reference's
    1-D RoPE table and temporal mask (the action temporal call)."""
    from multics_b200.action import get_temporal_block_causal_mask
    from multics_b200.attention import SelfAttention
    from multics_b200.rope import precompute_freqs_cis

    B, F, n, win, H, D = (int(x) for x in GOLD["temporal/shape"])
    sa = _load(SelfAttention(H * D, H, eps=1e-6), "temporal").cuda().bfloat16()
    x = _bf16(GOLD["temporal/x"]).reshape(B, F, H * D).cuda()
    freqs = precompute_freqs_cis(D, end=F).unsqueeze(1).cuda()
    mask = get_temporal_block_causal_mask(F, n, win, device="cuda")
    with torch.no_grad():
        out = sa(x, freqs, mask)
    _close(out, torch.from_numpy(GOLD["temporal/out"]).cuda(), "temporal module")


def test_keyboard_cross_attention_matches_reference_module():
    from multics_b200.action import get_temporal_block_causal_mask, keyboard_frame_mask
    from multics_b200.attention import CrossAttention

    P, F, n, win, L, K, H, D = (int(x) for x in GOLD["keyboard/shape"])
    ca = _load(CrossAttention(H * D, H, eps=1e-6), "keyboard").cuda().bfloat16()
    x = _bf16(GOLD["keyboard/x"]).reshape(P, F * L, H * D).cuda()
    ctx = _bf16(GOLD["keyboard/ctx"]).reshape(P, F * K, H * D).cuda()
    mask = keyboard_frame_mask(get_temporal_block_causal_mask(F, n, win, device="cuda"), L, K)
    with torch.no_grad():
        out = ca(x, ctx, mask)
    _close(out, torch.from_numpy(GOLD["keyboard/out"]).cuda(), "keyboard module")


@pytest.mark.parametrize("n,win", [(1, -1), (7, 24)])
def test_config3_temporal_full_size(n, win):
    """880 sequences (4 players x 220 patches) of 42 frames, 24 heads."""
    from multics_b200.action import get_temporal_block_causal_mask, shared_mask_attention
    from multics_b200.attention import device_error

    B, F, H = 880, 42, 24
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(B, F, H * 128, generator=g, device="cuda").bfloat16() for _ in range(3))
    m = get_temporal_block_causal_mask(F, n, win, device="cuda")
    out = shared_mask_attention(q, k, v, H, m)
    torch.cuda.synchronize()
    assert device_error() == 0
    for b0 in (0, 1, 2, 437, 877, 879):
        sl = slice(b0, b0 + 1)
        ref = R.shared_mask_sdpa(q[sl].float(), k[sl].float(), v[sl].float(), H, m)
        _close(out[sl], ref, ("temporal", b0))


def test_config3_keyboard_full_size():
    """4 players x (42 frames x 220 patches) queries over 42 x 12 keyboard
    tokens, the 1-frame block-causal frame mask repeated."""
    from multics_b200.action import (get_temporal_block_causal_mask, keyboard_frame_mask,
                                     shared_mask_attention)
    from multics_b200.attention import device_error

    P, F, L, K, H = 4, 42, 220, 12, 24
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(P, F * L, H * 128, generator=g, device="cuda").bfloat16()
    k, v = (torch.randn(P, F * K, H * 128, generator=g, device="cuda").bfloat16() for _ in range(2))
    m = keyboard_frame_mask(get_temporal_block_causal_mask(F, 1, -1, device="cuda"), L, K)
    out = shared_mask_attention(q, k, v, H, m)
    torch.cuda.synchronize()
    assert device_error() == 0
    for p in range(P):
        for r0 in (0, 20 * L, (F - 1) * L):
            rows = slice(r0, r0 + L)
            ref = R.shared_mask_sdpa(q[p:p + 1, rows].float(), k[p:p + 1].float(),
                                     v[p:p + 1].float(), H, m[rows])
            _close(out[p:p + 1, rows], ref, ("keyboard", p, r0))

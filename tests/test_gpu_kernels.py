"""GPU parity of the CUDA kernels against the reference goldens and the oracle.

* tcgen05 operand self-test against torch matmul;
* dense masks and Flex block lists: bit-exact with the reference;
* per-row key bitmasks of the attention plan: re-expanded, bit-exact with the
  reference dense mask;
* fused prologue: camera + RMSNorm + RoPE vs the reference fp32 values;
* attention: vs the reference fp32 output (max-abs <= 2e-2, cos >= 0.9995,
  the tolerance of the north-star spec) and vs a torch fp32 attention on
  larger random hierarchical configs.
"""

import math

import numpy as np
import pytest
import torch

from helpers import case_names, mask_case, num_case
from oracle import hier_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)


def _mask_args(c, dev):
    t = lambda a, dt: None if a is None else torch.as_tensor(np.asarray(a), dtype=dt, device=dev)  # noqa: E731
    return dict(
        group_labels=t(c["labels"], torch.long), active_group=t(c["active"], torch.bool),
        direct_player=c["direct"], device=dev, membership=t(c["membership"], torch.bool),
        global_only=t(c["global_only"], torch.bool), hier_no_local_hub=c["no_local"])


def _dims(c):
    return (c["P"], c["T"], c["L"], c["N"], c["KL"], c["KG"], c["n"], c["win"])


def test_umma_operand_selftest(dev):
    from multics_b200 import _lib
    from multics_b200._lib import ptr, stream_ptr

    g = torch.Generator(device="cpu").manual_seed(1)
    a = torch.randn(128, 128, generator=g).to(torch.bfloat16).to(dev)
    b = torch.randn(128, 128, generator=g).to(torch.bfloat16).to(dev)
    outs = [torch.zeros(128, 128, device=dev) for _ in range(3)]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().hier_selftest_umma(ptr(a), ptr(b), *map(ptr, outs), ptr(err), stream_ptr()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    af, bf = a.float(), b.float()
    torch.testing.assert_close(outs[0], af @ bf.T, atol=1e-2, rtol=1e-3)
    torch.testing.assert_close(outs[1], af @ bf, atol=1e-2, rtol=1e-3)
    torch.testing.assert_close(outs[2], af @ bf, atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("name", case_names("mask"))
def test_dense_mask_bit_exact(dev, name):
    from multics_b200.hier_masks import build_stage2_hier_self_attn_mask

    c = mask_case(name)
    m = build_stage2_hier_self_attn_mask(*_dims(c), **_mask_args(c, dev))
    assert torch.equal(m.cpu(), torch.from_numpy(c["dense"]))


@pytest.mark.parametrize("name", case_names("mask"))
def test_block_mask_lists_bit_exact(dev, name):
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask, clear_block_mask_cache

    clear_block_mask_cache()
    c = mask_case(name)
    bm, S, S_pad = build_stage2_hier_flex_block_mask(*_dims(c), **_mask_args(c, dev))
    assert (S, S_pad) == (c["S"], c["S_pad"])
    assert np.array_equal(bm.kv_num_blocks.flatten().cpu().numpy(), c["kv_num_blocks"])
    assert np.array_equal(bm.kv_flat.cpu().numpy(), c["kv_indices"])
    assert np.array_equal(bm.full_kv_num_blocks.flatten().cpu().numpy(), c["full_kv_num_blocks"])
    assert np.array_equal(bm.full_flat.cpu().numpy(), c["full_kv_indices"])


def expand_plan(bm):
    """Dense [S,S] mask implied by an attention plan (query pairs, key tiles,
    per-half mask selectors, row bitmasks)."""
    S = bm.S
    qp = bm.q_pairs.cpu().numpy()
    kv = bm.kv_tiles.cpu().numpy()
    rm = bm.row_masks.cpu().numpy().view(np.uint32)
    dense = np.zeros((S, S + 256), bool)
    for q0, qn0, q1, qn1, b, e, _, _ in qp:
        for j in range(b, e):
            k0, k1, m0, m1 = kv[j]
            for qs, qn, mi in ((q0, qn0, m0), (q1, qn1, m1)):
                if mi == -2 or qn == 0:
                    continue
                if mi == -1:
                    bits = np.ones((128, 128), bool)
                else:
                    w = rm[mi]
                    bits = ((w[:, np.arange(128) // 32] >> (np.arange(128) % 32)) & 1).astype(bool)
                dense[qs:qs + qn, k0:k0 + 64] |= bits[:qn, :64]
                dense[qs:qs + qn, k1:k1 + 64] |= bits[:qn, 64:]
    return dense[:, :S]


@pytest.mark.parametrize("name", case_names("mask"))
def test_plan_row_masks_reproduce_dense_mask(dev, name):
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask, clear_block_mask_cache

    clear_block_mask_cache()
    c = mask_case(name)
    bm, _, _ = build_stage2_hier_flex_block_mask(*_dims(c), **_mask_args(c, dev))
    assert np.array_equal(expand_plan(bm), c["dense"])
    order = bm.order.cpu().numpy()
    assert sorted(order.tolist()) == list(range(bm.num_pairs))
    assert int(bm.n_kv_tiles.item()) == int(bm.q_pairs[:, 5].max().item())


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-30))


@pytest.mark.parametrize("name", [n for n in case_names("num") if "d128" in n])
def test_prologue_matches_reference(dev, name):
    from multics_b200.attention import hier_prep_qk

    d = num_case(name)
    m = d["meta"]
    bf = lambda k: torch.from_numpy(d[k + "_bits"].view(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
    freqs = torch.from_numpy(d["freqs"]).to(dev)
    q, k = hier_prep_qk(bf("qx"), bf("kx"), freqs, m["H"], norm_q_weight=bf("nqw"),
                        norm_k_weight=bf("nkw"), cam_tokens=bf("cam"), cam_q_weight=bf("wcq"),
                        cam_k_weight=bf("wck"))
    torch.cuda.synchronize()
    for got, ref in ((q, d["roped_q"]), (k, d["roped_k"])):
        ref = torch.from_numpy(ref).to(dev)
        err = (got.float() - ref).abs()
        assert float(err.max()) <= 0.02 * float(ref.abs().max())
        assert _cos(got.float(), ref) >= 0.9999


@pytest.mark.parametrize("name", [n for n in case_names("num") if "d128" in n])
def test_layer_matches_reference_fp32(dev, name):
    """Full hot path (prologue + attention) vs the reference fp32 output."""
    from multics_b200.attention import attention_from_plan, hier_prep_qk
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask

    d = num_case(name)
    m = d["meta"]
    bf = lambda k: torch.from_numpy(d[k + "_bits"].view(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
    q, k = hier_prep_qk(bf("qx"), bf("kx"), torch.from_numpy(d["freqs"]).to(dev), m["H"],
                        norm_q_weight=bf("nqw"), norm_k_weight=bf("nkw"), cam_tokens=bf("cam"),
                        cam_q_weight=bf("wcq"), cam_k_weight=bf("wck"))
    if m["membership"]:
        kw = dict(group_labels=None, active_group=None,
                  membership=torch.from_numpy(d["membership"]).to(dev),
                  global_only=torch.from_numpy(d["global_only"]).to(dev))
    else:
        kw = dict(group_labels=torch.from_numpy(d["labels"]).to(dev), active_group=None)
    bm, S, _ = build_stage2_hier_flex_block_mask(m["P"], m["T"], m["L"], m["N"], m["KL"], m["KG"],
                                                 m["n"], m["win"], direct_player=True, device=dev,
                                                 **kw)
    out = attention_from_plan(q, k, bf("v"), bm, m["H"])
    torch.cuda.synchronize()
    ref = torch.from_numpy(d["out"]).to(dev)
    assert torch.isfinite(out).all()
    assert float((out.float() - ref).abs().max()) <= MAX_ABS
    assert _cos(out.float(), ref) >= MIN_COS


def torch_masked_attention(q, k, v, mask, H):
    """Plain PyTorch fp32 reference: softmax(q k^T / sqrt(D) + mask) v per head."""
    S, dim = q.shape
    D = dim // H
    qf, kf, vf = (t.float().view(-1, H, D).transpose(0, 1) for t in (q, k, v))
    s = qf @ kf.transpose(1, 2) / math.sqrt(D)
    s = s.masked_fill(~mask[None], float("-inf"))
    p = torch.softmax(s, -1)
    p = torch.nan_to_num(p, nan=0.0)
    return (p @ vf).transpose(0, 1).reshape(S, dim)


RANDOM_CASES = [
    # P, T, L, N, KL, KG, n, win, mode
    (4, 6, 50, 2, 4, 3, 1, -1, "labels"),
    (4, 6, 50, 2, 4, 3, 3, 4, "labels"),
    (5, 4, 37, 3, 5, 6, 2, 2, "membership"),
    (3, 5, 130, 2, 16, 6, 1, -1, "labels"),
]


@pytest.mark.parametrize("case", RANDOM_CASES)
def test_attention_random_configs_vs_torch_fp32(dev, case):
    from multics_b200.attention import attention_from_plan
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask

    P, T, L, N, KL, KG, n, win, mode = case
    H = 2
    g = torch.Generator().manual_seed(hash(case) & 0xFFFF)
    S = P * T * L + T * (N * KL + KG)
    q, k, v = (torch.randn(S, H * 128, generator=g).mul(0.5).to(torch.bfloat16).to(dev)
               for _ in range(3))
    if mode == "labels":
        labels = torch.randint(0, N, (T, P), generator=g)
        for t0 in range(0, T, n):
            labels[t0:t0 + n] = labels[t0]
        kw = dict(group_labels=labels.to(dev), active_group=None)
        okw = dict(labels=labels.numpy(), direct=True)
    else:
        mem = torch.rand(T, N, P, generator=g) < 0.4
        go = ~mem.any(1)
        mem[:, N - 1] = False  # an empty slot: inactive local hub rows
        kw = dict(group_labels=None, active_group=None, membership=mem.to(dev), global_only=go.to(dev))
        okw = dict(membership=mem.numpy(), global_only=go.numpy(), direct=True)
    bm, _, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, n, win, direct_player=True,
                                                 device=dev, **kw)
    out = attention_from_plan(q, k, v, bm, H)
    mask = torch.from_numpy(O.dense_mask(P, T, L, N, KL, KG, n, win, **okw)).to(dev)
    ref = torch_masked_attention(q, k, v, mask, H)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert float((out.float() - ref).abs().max()) <= MAX_ABS
    assert _cos(out.float(), ref) >= MIN_COS


SEQUENCE_CASES = [c for c in RANDOM_CASES if c[-1] == "labels"] + [
    (3, 4, 70, 3, 5, 6, 2, -1, "labels"),   # a group idle in some frames
    (2, 12, 40, 2, 16, 6, 1, -1, "labels"),  # several 128-row hub tiles per group
]


@pytest.mark.parametrize("case", SEQUENCE_CASES)
def test_sequence_plan_random_configs_vs_torch_fp32(dev, case):
    """The sequence plan (player-frame pairs, group tiles of hub queries) on
    roped q/k permuted into its row order; output rows return to the
    sequence order."""
    from multics_b200.attention import sequence_plan
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask

    P, T, L, N, KL, KG, n, win, _ = case
    H = 2
    g = torch.Generator().manual_seed(hash(case) & 0xFFFF)
    S = P * T * L + T * (N * KL + KG)
    q, k, v = (torch.randn(S, H * 128, generator=g).mul(0.5).to(torch.bfloat16).to(dev)
               for _ in range(3))
    labels = torch.randint(0, N, (T, P), generator=g)
    for t0 in range(0, T, n):
        labels[t0:t0 + n] = labels[t0]
    bm, _, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, n, win, labels.to(dev), None,
                                                 True, dev)
    sp = sequence_plan(bm, H)
    assert sp is not None
    src = sp.plan_to_seq.long()
    out = sp.attend(q[src].contiguous(), k[src].contiguous(), v)
    mask = torch.from_numpy(O.dense_mask(P, T, L, N, KL, KG, n, win, labels=labels.numpy(),
                                         direct=True)).to(dev)
    ref = torch_masked_attention(q, k, v, mask, H)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert float((out.float() - ref).abs().max()) <= MAX_ABS
    assert _cos(out.float(), ref) >= MIN_COS


def test_sequence_plan_caller_active_groups(dev):
    """Caller-given active groups: an active group without members (its hub
    rows attend to hub tokens only) and an inactive group with members (its
    hub rows attend to themselves, players do not see them)."""
    from multics_b200.attention import sequence_plan
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask

    P, T, L, N, KL, KG, H = 4, 4, 40, 3, 4, 3, 2
    labels = torch.tensor([[0, 0, 1, 1]] * T)
    active = torch.tensor([[True, True, True], [True, False, True], [True, True, False],
                           [False, True, True]])
    g = torch.Generator().manual_seed(11)
    S = P * T * L + T * (N * KL + KG)
    q, k, v = (torch.randn(S, H * 128, generator=g).mul(0.5).to(torch.bfloat16).to(dev)
               for _ in range(3))
    bm, _, _ = build_stage2_hier_flex_block_mask(P, T, L, N, KL, KG, 1, -1, labels.to(dev),
                                                 active.to(dev), True, dev)
    sp = sequence_plan(bm, H)
    assert sp is not None
    src = sp.plan_to_seq.long()
    out = sp.attend(q[src].contiguous(), k[src].contiguous(), v)
    mask = torch.from_numpy(O.dense_mask(P, T, L, N, KL, KG, 1, -1, labels=labels.numpy(),
                                         active=active.numpy(), direct=True)).to(dev)
    ref = torch_masked_attention(q, k, v, mask, H)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert float((out.float() - ref).abs().max()) <= MAX_ABS
    assert _cos(out.float(), ref) >= MIN_COS


@pytest.mark.parametrize("plan", ["segments", "blocks"])
@pytest.mark.parametrize("name", [n for n in case_names("num") if "d128" in n])
def test_layer_entry_matches_reference_fp32(dev, name, plan, monkeypatch):
    """hier_attention_layer (prologue + attention through the plan the entry
    point picks) vs the reference fp32 output, with either work plan."""
    from multics_b200.attention import FULL_SEQUENCE_PLAN_ENV, hier_attention_layer
    from multics_b200.hier_masks import build_stage2_hier_flex_block_mask

    monkeypatch.setenv(FULL_SEQUENCE_PLAN_ENV, plan)
    d = num_case(name)
    m = d["meta"]
    bf = lambda k: torch.from_numpy(d[k + "_bits"].view(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
    if m["membership"]:
        kw = dict(group_labels=None, active_group=None,
                  membership=torch.from_numpy(d["membership"]).to(dev),
                  global_only=torch.from_numpy(d["global_only"]).to(dev))
    else:
        kw = dict(group_labels=torch.from_numpy(d["labels"]).to(dev), active_group=None)
    bm, S, _ = build_stage2_hier_flex_block_mask(m["P"], m["T"], m["L"], m["N"], m["KL"], m["KG"],
                                                 m["n"], m["win"], direct_player=True, device=dev,
                                                 **kw)
    out = hier_attention_layer(bf("qx"), bf("kx"), bf("v"), torch.from_numpy(d["freqs"]).to(dev),
                               bm, m["H"], norm_q_weight=bf("nqw"), norm_k_weight=bf("nkw"),
                               cam_tokens=bf("cam"), cam_q_weight=bf("wcq"),
                               cam_k_weight=bf("wck"))
    torch.cuda.synchronize()
    ref = torch.from_numpy(d["out"]).to(dev)
    assert torch.isfinite(out).all()
    assert float((out.float() - ref).abs().max()) <= MAX_ABS
    assert _cos(out.float(), ref) >= MIN_COS


def test_paged_pool_matches_contiguous(dev):
    """Keys/values scattered over shuffled 64-token pages give identical output."""
    from multics_b200.attention import attention_from_plan
    from multics_b200.hier_masks import build_block_plan, make_grouping_spec

    P, T, L, N, KL, KG, H = 4, 6, 50, 2, 4, 3, 2
    g = torch.Generator().manual_seed(5)
    S = P * T * L + T * (N * KL + KG)
    q, k, v = (torch.randn(S, H * 128, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    labels = torch.tensor([[0, 0, 1, 1]] * T, device=dev)
    spec = make_grouping_spec(P, T, L, N, KL, KG, 1, -1, labels, None, True, dev)
    base = build_block_plan(spec)
    n_pages = (S + 63) // 64
    perm = torch.randperm(n_pages, generator=g)
    kp = torch.zeros(n_pages * 64, H * 128, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    for logical in range(n_pages):
        r0, r1 = logical * 64, min(S, logical * 64 + 64)
        phys = int(perm[logical])
        kp[phys * 64: phys * 64 + (r1 - r0)] = k[r0:r1]
        vp[phys * 64: phys * 64 + (r1 - r0)] = v[r0:r1]
    paged = build_block_plan(spec, page_table=perm.to(torch.int32))
    o1 = attention_from_plan(q, k, v, base, H)
    o2 = attention_from_plan(q, kp, vp, paged, H)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("name", case_names("mask"))
def test_dense_mask_block_plan_bit_exact(dev, name):
    """The block plan built from the reference's dense mask bytes has the
    Flex block lists of the reference and re-expands to the same mask."""
    from multics_b200.hier_masks import build_dense_block_plan

    c = mask_case(name)
    bm = build_dense_block_plan(torch.from_numpy(c["dense"]).to(dev), c["S"])
    assert bm.S_pad == c["S_pad"]
    assert np.array_equal(bm.kv_num_blocks.flatten().cpu().numpy(), c["kv_num_blocks"])
    assert np.array_equal(bm.kv_flat.cpu().numpy(), c["kv_indices"])
    assert np.array_equal(bm.full_kv_num_blocks.flatten().cpu().numpy(), c["full_kv_num_blocks"])
    assert np.array_equal(bm.full_flat.cpu().numpy(), c["full_kv_indices"])
    assert np.array_equal(expand_plan(bm), c["dense"])

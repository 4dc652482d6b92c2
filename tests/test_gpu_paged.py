"""Paged key/value pools on the sequence plan (benchmark configuration 5:
64-token pages, page table shuffled by seed; the reference's paged KV layout,
multics/models/kernels/hier_paged_attention.py:209-260).  The player rows'
keys and values live in 64-row pages at shuffled physical positions; the plan
covers each pair's keys page by page.  A shuffled table must give the same
bits as the identity table (the same tiles, other physical rows), and both
must match the fp32 reference."""

import numpy as np
import pytest
import torch

from oracle import hier_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


def _layer(P, T, h, w, N, KL, KG, H, labels, page_table, seed=3, n_block=1, win=-1):
    from multics_b200.attention import HierSequencePlan, hier_prep_qk
    from multics_b200.hier_masks import make_grouping_spec

    L, dim = h * w, H * 128
    S = P * T * L + T * (N * KL + KG)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    qx, kx, v = ((torch.randn(S, dim, generator=g) * 0.5).to(torch.bfloat16) for _ in range(3))
    cam = torch.zeros(S, 12)
    cam[:P * T * L] = torch.randn(P * T, 12, generator=g).repeat_interleave(L, 0)
    cam = cam.to(torch.bfloat16)
    wcq, wck = ((torch.randn(dim, 12, generator=g) * 0.02).to(torch.bfloat16) for _ in range(2))
    nqw, nkw = ((1 + 0.02 * torch.randn(dim, generator=g)).to(torch.bfloat16) for _ in range(2))
    freqs = O.self_attn_freqs_with_hub(P, T, h, w, N * KL + KG, 128, (12, 32, 42, 42), 10)
    spec = make_grouping_spec(P, T, L, N, KL, KG, n_block, win, torch.tensor(labels, device=dev),
                              None, True, dev)
    sp = HierSequencePlan(spec, H, page_table=page_table)
    assert int(sp.core.status.item()) == 0
    q_plan = torch.empty(S, dim, dtype=torch.bfloat16, device=dev)
    k_pool = torch.empty(sp.pool_size, dim, dtype=torch.bfloat16, device=dev)
    ft = torch.from_numpy(freqs).float().to(dev)
    hier_prep_qk(qx.to(dev), kx.to(dev), ft, H, norm_q_weight=nqw.to(dev),
                 norm_k_weight=nkw.to(dev), cam_tokens=cam.to(dev), cam_q_weight=wcq.to(dev),
                 cam_k_weight=wck.to(dev), out=(q_plan, k_pool), out_rows=sp.seq_to_plan,
                 k_out_rows=sp.pool_rows)
    v_pool = sp.to_pool(v.to(dev))
    out = sp.attend_paged(q_plan, k_pool, v_pool)
    torch.cuda.synchronize()
    f32 = lambda t: t.float().numpy()  # noqa: E731
    qr, kr = O.prologue(f32(qx), f32(kx), f32(cam), f32(wcq), f32(wck), f32(nqw), f32(nkw),
                        freqs, H)
    return out, (qr, kr, f32(v)), S


@pytest.mark.parametrize("shape", [(3, 5, 4, 8, 2, 4, 3, 2), (4, 6, 5, 9, 2, 8, 6, 2)])
def test_paged_sequence_plan(shape):
    P, T, h, w, N, KL, KG, H = shape
    L = h * w
    rng = np.random.default_rng(7)
    labels = np.array([[p * N // P for p in range(P)]] * T)
    n_pages = -(-P * T * L // 64) + 3  # a few spare physical pages
    ident = np.arange(n_pages)
    shuf = rng.permutation(n_pages)
    out_i, (qr, kr, v), S = _layer(P, T, h, w, N, KL, KG, H, labels, ident)
    out_s, _, _ = _layer(P, T, h, w, N, KL, KG, H, labels, shuf)
    assert torch.equal(out_i, out_s)
    dense = O.dense_mask(P, T, L, N, KL, KG, 1, -1, labels=labels, direct=True)
    ref = O.masked_attention(qr, kr, v, H, lambda a, b: dense[a:b])
    got = out_s.float().cpu().numpy()
    err = float(np.abs(got - ref).max())
    cos = float((got * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err <= MAX_ABS, err
    assert cos >= MIN_COS, cos


def test_paged_plan_refuses_short_table():
    from multics_b200.attention import HierSequencePlan
    from multics_b200.hier_masks import make_grouping_spec

    dev = torch.device("cuda")
    spec = make_grouping_spec(2, 3, 40, 1, 4, 2, 1, -1, torch.zeros(3, 2, dtype=torch.long,
                                                                      device=dev), None, True, dev)
    with pytest.raises(ValueError):
        HierSequencePlan(spec, 2, page_table=np.arange(2))

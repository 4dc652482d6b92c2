"""Pin the timed CPU baseline (the reference's CPU path issued as torch calls,
``oracle/ref_cpu_path.py``) against the reference's own recorded outputs, and
its unit-expanded dense mask against the token-level oracle mask."""

import numpy as np
import pytest
import torch

from helpers import case_names, mask_case, mask_kwargs, num_case
from oracle import hier_oracle as O
from oracle import ref_cpu_path as R


@pytest.mark.parametrize("name", case_names("num"))
def test_torch_reference_path_matches_reference_outputs(name):
    c = num_case(name)
    m = c["meta"]
    H, S = m["H"], m["S"]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).float()  # noqa: E731
    fr = torch.from_numpy(c["freqs"])
    freqs = torch.view_as_complex(fr.contiguous()).unsqueeze(1)
    q, k = R.prologue(t(c["qx"])[None], t(c["kx"])[None], t(c["cam"])[None], t(c["wcq"]),
                      t(c["wck"]), t(c["nqw"]), t(c["nkw"]), freqs, H)
    np.testing.assert_allclose(q[0].numpy(), c["roped_q"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(k[0].numpy(), c["roped_k"], atol=1e-5, rtol=1e-5)
    kw = dict(labels=None if "membership" in c else c["labels"], direct=True,
              membership=c.get("membership"), global_only=c.get("global_only"))
    mask = O.dense_mask(m["P"], m["T"], m["L"], m["N"], m["KL"], m["KG"], m["n"], m["win"],
                        **kw)
    assert int(mask.sum()) == int(c["mask_popcount"])
    o = R.sdpa_rows(q, k, t(c["v"])[None], torch.from_numpy(mask), H)
    np.testing.assert_allclose(o[0].numpy(), c["out"], atol=2e-5, rtol=1e-4)
    # a row chunk of a subset of heads is the same slice of the whole output
    D = m["D"]
    part = R.sdpa_rows(q, k, t(c["v"])[None], torch.from_numpy(mask[40:97]), H, heads=[1],
                       r0=40, r1=97)
    np.testing.assert_allclose(part[0].numpy(), c["out"][40:97, D:2 * D], atol=2e-5, rtol=1e-4)


@pytest.mark.parametrize("name", case_names("mask"))
def test_unit_expanded_mask_equals_token_mask(name):
    c = mask_case(name)
    um = R.UnitMask(c["P"], c["T"], c["L"], c["N"], c["KL"], c["KG"], c["n"], c["win"],
                    **mask_kwargs(c))
    S = c["dense"].shape[0]
    assert um.S == S
    got = np.concatenate([um.rows(r, min(S, r + 61)) for r in range(0, S, 61)])
    assert np.array_equal(got, c["dense"])


def test_unit_expanded_mask_full_size_rows():
    """Rows of the config-2 mask by unit expansion equal the token-level oracle."""
    from multics_b200.synth import CONFIGS

    cfg = CONFIGS["cfg2"]
    lab = np.array([cfg.groups] * cfg.T)
    um = R.UnitMask(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG, 1, -1, labels=lab, direct=True)
    for r0 in (0, 20000, cfg.S - 300):
        ref = O.dense_mask(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG, 1, -1, labels=lab,
                           direct=True, rows=slice(r0, r0 + 300))
        assert np.array_equal(um.rows(r0, r0 + 300), ref)

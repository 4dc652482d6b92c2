"""Generate golden fixtures for the hierarchical group-attention hot path.

This script imports the reference implementation (TencentARC/Multics, pure
Python/PyTorch) from a local checkout and records its outputs on small seeded
inputs.  It is run once in a container that has the reference checkout; the
resulting ``*.npz`` files are committed next to this script and are what the
tests read (the reference itself is not available where the GPU tests run).

Usage::

    python tests/golden/gen_golden.py --reference <path-to-Multics-checkout>

Fixtures written (all under ``tests/golden``):

* ``masks.npz``      dense masks (``build_stage2_hier_self_attn_mask``,
  ``multics/models/hier_masks.py:364-641``) and Flex BlockMask block lists
  (``build_stage2_hier_flex_block_mask``, ``hier_masks.py:722-1149``) for
  labels / membership / no-local / dynamic-grouping cases, including the
  reference's own test inputs and its real grouping fixtures.
* ``segmented.npz``  ``_build_metadata`` outputs
  (``multics/models/kernels/hier_segmented_attention.py:156-395``) and the
  varlen plans derived from them (``hier_packed_attention.py:32-102``).
* ``tiled.npz``      ``build_hier_tiled_full_sequence_layouts`` /
  ``build_hier_tiled_cached_layout`` (``hier_tiled_attention.py:244-655``).
* ``causal.npz``     ``SelfAttention.causal_forward_hier_hub``
  (``multics/models/attention.py:456-1005``) over consecutive blocks with
  rolling caches: per-block inputs and outputs, final cache contents.
* ``action.npz``     the action branch's masks (``get_temporal_block_causal_mask``,
  ``hier_masks.py:1152-1166``, and its keyboard repeat, ``blocks.py:446-448``)
  and fp32 outputs of the reference's ``SelfAttention`` over a batch of
  frame sequences (the per-frame action attention, ``blocks.py:677-691``) and
  of its ``CrossAttention`` under the keyboard mask (``blocks.py:692-697``).
* ``grads.npz``      gradients, by the reference's own autograd, of the
  reference attention path (camera add, RMSNorm, float64 RoPE, masked SDPA;
  ``attention.py:307-320,231-242``, ``rope.py:248-254``, ``attention.py:39-54``)
  with respect to its inputs and the camera / norm weights, for a seeded
  output gradient, on the config-1 head_dim-128 cases of ``numerics.npz``.
* ``numerics.npz``   fp32 outputs of the reference attention path
  (camera Q/K add ``attention.py:307-320``, RMSNorm ``:231-242``, float64
  RoPE ``rope.py:248-254``, masked SDPA ``attention.py:39-54``) on seeded
  inputs, for head_dim 64 (config 1 as stated) and head_dim 128.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _setup(reference: str):
    os.environ.setdefault("WAN_HIER_BLOCKMASK_COMPILE", "0")
    sys.path.insert(0, reference)
    import torch  # noqa: F401
    import multics.models.attention as attn_mod

    # With a mask the reference always routes through SDPA, but its unmasked
    # helpers would pick an installed flash-attn wheel (CUDA only) otherwise.
    attn_mod.FLASH_ATTN_2_AVAILABLE = False
    attn_mod.FLASH_ATTN_3_AVAILABLE = False
    attn_mod.SAGE_ATTN_AVAILABLE = False
    return attn_mod


# ---------------------------------------------------------------------------
# mask cases
# ---------------------------------------------------------------------------


def _mask_cases(reference: str):
    import torch

    cases = []

    def add(name, P, T, L, N, KL, KG, n, win, direct, labels=None, membership=None,
            global_only=None, active=None, no_local=False):
        cases.append(
            dict(name=name, P=P, T=T, L=L, N=N, KL=KL, KG=KG, n=n, win=win,
                 direct=bool(direct), labels=labels, membership=membership,
                 global_only=global_only, active=active, no_local=bool(no_local))
        )

    # Config 1 of the benchmark plan (frame-segmented causal, n=1, window -1).
    lab = torch.tensor([[0, 0, 1, 1]] * 3)
    add("cfg1_n1", 4, 3, 16, 2, 8, 6, 1, -1, True, labels=lab)
    add("cfg1_n1_nodirect", 4, 3, 16, 2, 8, 6, 1, -1, False, labels=lab)
    add("cfg1_n3_w21", 4, 3, 16, 2, 8, 6, 3, 21, True, labels=lab)
    # Reference tiled-layout test inputs (tests/test_hier_tiled_layout.py:211-233).
    lab9 = torch.tensor(
        [[0, 0, 1, 1]] * 3 + [[0, 2, 2, 0]] * 3 + [[1, 1, 2, 2]] * 3, dtype=torch.long
    )
    act9 = torch.zeros(9, 3, dtype=torch.bool)
    act9.scatter_(1, lab9, True)
    add("tiled_test_direct", 4, 9, 7, 3, 2, 3, 3, 4, True, labels=lab9, active=act9)
    add("tiled_test_nodirect", 4, 9, 7, 3, 2, 3, 3, 4, False, labels=lab9, active=act9)
    # Explicit active with an inactive slot -> inactive-local self edges.
    act_off = act9.clone()
    act_off[3:6, 1] = False
    add("inactive_slot", 4, 9, 7, 3, 2, 3, 3, 4, True, labels=lab9, active=act_off)
    # Membership cases (tests/test_hier_flexible_membership_mask.py:180-266).
    T = 3
    mem = torch.zeros(T, 2, 4, dtype=torch.bool)
    mem[:, 0, 1] = True
    mem[:, 0, 2] = True
    go = torch.zeros(T, 4, dtype=torch.bool)
    go[:, 0] = True
    go[:, 3] = True
    add("mem_p4_mixed", 4, 3, 2, 2, 1, 1, 3, 7, True, membership=mem, global_only=go)
    add("mem_p4_allgo", 4, 3, 2, 2, 1, 1, 3, 7, True,
        membership=torch.zeros(T, 2, 4, dtype=torch.bool),
        global_only=torch.ones(T, 4, dtype=torch.bool))
    mem10 = torch.zeros(T, 4, 10, dtype=torch.bool)
    mem10[:, 0, 0] = True
    mem10[:, 1, 0] = True
    mem10[:, 0, 1] = True
    mem10[:, 1, 2] = True
    go10 = torch.zeros(T, 10, dtype=torch.bool)
    go10[:, 3] = True
    add("mem_p10_anchor", 10, 3, 2, 4, 1, 1, 3, 7, True, membership=mem10, global_only=go10)
    # No-local topology (K_L = 0), labels and membership.
    add("nolocal_labels", 4, 4, 5, 2, 0, 3, 2, 3, True,
        labels=torch.tensor([[0, 0, 1, 1]] * 4), no_local=True)
    add("nolocal_mem", 4, 3, 2, 2, 0, 2, 3, 7, True, membership=mem, global_only=go,
        no_local=True)
    # Dynamic grouping: 8 players in 4 groups of 2, re-permuted every 3 frames.
    g = torch.Generator().manual_seed(0)
    rows = []
    for blk in range(2):
        perm = torch.randperm(8, generator=g)
        row = torch.empty(8, dtype=torch.long)
        row[perm] = torch.arange(8) // 2
        rows += [row] * 3
    add("dyn_p8", 8, 6, 5, 4, 2, 2, 3, 21, True, labels=torch.stack(rows))
    add("dyn_p8_n1", 8, 6, 5, 4, 2, 2, 1, -1, True, labels=torch.stack(rows))
    # Uneven groups (3,3,2,2), 10 players, labels.
    lab10 = torch.tensor([0, 0, 0, 1, 1, 1, 2, 2, 3, 3])
    add("uneven_p10", 10, 4, 3, 4, 2, 2, 1, -1, True, labels=lab10[None].repeat(4, 1))
    # Real grouping fixtures shipped with the reference.
    ref = Path(reference)
    for stem, P, N in (("p4_round_start", 4, 2), ("p6_moving_pairs", 6, 3),
                       ("p10_moving_pairs", 10, 4)):
        d = np.load(ref / "tests/fixtures/grouping" / f"{stem}.labels.npz")
        memf = torch.from_numpy(d["membership"].astype(bool))
        gof = torch.from_numpy(d["global_only"].astype(bool))
        add(f"fixture_{stem}", P, memf.shape[0], 2, N, 1, 2, 3, 21, True,
            membership=memf, global_only=gof)
    grp = torch.load(ref / "asset/examples/4players/4_01/groups.pt")
    add("asset_4_01", 4, grp["membership"].shape[0], 2, 2, 2, 2, 3, 21, True,
        membership=grp["membership"].bool(), global_only=grp["global_only"].bool())
    return cases


def gen_masks(reference: str, out: dict):
    import torch
    from multics.models.hier_masks import (
        build_stage2_hier_flex_block_mask,
        build_stage2_hier_self_attn_mask,
    )

    names = []
    for c in _mask_cases(reference):
        P, T, L, N, KL, KG = (c[k] for k in ("P", "T", "L", "N", "KL", "KG"))
        labels = c["labels"]
        if labels is None:
            labels_arg = torch.zeros(T, P, dtype=torch.long)
        else:
            labels_arg = labels
        kw = dict(
            group_labels=labels_arg,
            active_group=c["active"],
            direct_player=c["direct"],
            device=torch.device("cpu"),
            membership=c["membership"],
            global_only=c["global_only"],
            hier_no_local_hub=c["no_local"],
        )
        dense = build_stage2_hier_self_attn_mask(
            P, T, L, N, KL, KG, c["n"], c["win"], **kw
        )
        bm, S, S_pad = build_stage2_hier_flex_block_mask(
            P, T, L, N, KL, KG, c["n"], c["win"], **kw
        )
        nm = c["name"]
        names.append(nm)
        meta = {k: c[k] for k in ("P", "T", "L", "N", "KL", "KG", "n", "win", "direct",
                                  "no_local")}
        meta["mode"] = "membership" if c["membership"] is not None else "labels"
        meta["S"] = int(S)
        meta["S_pad"] = int(S_pad)
        out[f"{nm}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        out[f"{nm}/labels"] = labels_arg.numpy().astype(np.int64)
        if c["active"] is not None:
            out[f"{nm}/active"] = c["active"].numpy().astype(bool)
        if c["membership"] is not None:
            out[f"{nm}/membership"] = c["membership"].numpy().astype(bool)
            out[f"{nm}/global_only"] = c["global_only"].numpy().astype(bool)
        d = dense.numpy().astype(bool)
        out[f"{nm}/dense_bits"] = np.packbits(d, axis=None)
        out[f"{nm}/dense_popcount"] = np.array(int(d.sum()), dtype=np.int64)
        kvn = bm.kv_num_blocks[0, 0].numpy().astype(np.int32)
        kvi = bm.kv_indices[0, 0].numpy().astype(np.int32)
        fn = bm.full_kv_num_blocks[0, 0].numpy().astype(np.int32)
        fi = bm.full_kv_indices[0, 0].numpy().astype(np.int32)
        out[f"{nm}/kv_num_blocks"] = kvn
        out[f"{nm}/kv_indices"] = np.concatenate([kvi[r, : kvn[r]] for r in range(len(kvn))])
        out[f"{nm}/full_kv_num_blocks"] = fn
        out[f"{nm}/full_kv_indices"] = np.concatenate([fi[r, : fn[r]] for r in range(len(fn))])
    out["mask_case_names"] = np.frombuffer(json.dumps(names).encode(), dtype=np.uint8)


# ---------------------------------------------------------------------------
# segmented metadata + varlen plans
# ---------------------------------------------------------------------------


def _seg_cases():
    cases = []
    # tests/test_hier_segmented_metadata.py:111-152
    for P in (2, 4, 6, 8):
        for direct in (False, True):
            N = max(2, P // 2 + 1)
            L, KL, KG = 3, 2, 2
            n_frames, n_block, local_attn = 2, 2, 4
            frames = tuple(range(1, 7))
            labels_row = tuple(player % (N - 1) for player in range(P))
            active_row = tuple(group in labels_row for group in range(N))
            cases.append(dict(
                name=f"reftest_P{P}_d{int(direct)}", P=P, N=N, L=L, KL=KL, KG=KG,
                n_frames=n_frames, n_block=n_block, local_attn=local_attn,
                agent=tuple(frames for _ in range(P)), local=tuple(frames for _ in range(N)),
                glob=frames,
                local_active=tuple(tuple((f + g) % 3 != 0 and active_row[g] for f in frames)
                                   for g in range(N)),
                labels=(labels_row,) * n_frames, q_active=(active_row,) * n_frames,
                direct=direct, block_m=16, membership=None, global_only=None, no_local=False))
    # Released cached config shape with a reduced L (P=4, n=3, 24 retained
    # frames, window 21, K_L=5, K_G=6).
    fr = tuple(range(0, 24))
    cases.append(dict(
        name="cached_released", P=4, N=2, L=20, KL=5, KG=6, n_frames=3, n_block=3,
        local_attn=21, agent=(fr,) * 4, local=(fr,) * 2, glob=fr,
        local_active=((True,) * 24, tuple(f % 5 != 1 for f in fr)),
        labels=((0, 0, 1, 1),) * 3, q_active=((True, True),) * 3, direct=True,
        block_m=16, membership=None, global_only=None, no_local=False))
    # Membership + global_only (tests/test_hier_paged_attention.py:59-82 shape),
    # two cached blocks (frames 0..1 then 0..3).
    for tag, fr in (("blk0", (0, 1)), ("blk1", (0, 1, 2, 3))):
        T = 4
        mem = [[[False] * 4 for _ in range(2)] for _ in range(T)]
        for t in range(T):
            mem[t][0][0] = mem[t][0][1] = True
            mem[t][1][2] = True
        go = [[False, False, False, True] for _ in range(T)]
        cases.append(dict(
            name=f"membership_{tag}", P=4, N=2, L=8, KL=2, KG=2, n_frames=2, n_block=2,
            local_attn=4, agent=(fr,) * 4, local=(fr,) * 2, glob=fr,
            local_active=(tuple(True for _ in fr), tuple(True for _ in fr)),
            labels=None, q_active=((True, True),) * 2, direct=True, block_m=8,
            membership=mem, global_only=go, no_local=False))
    # Anchor player in two slots + an empty slot.
    T = 3
    mem = [[[False] * 5 for _ in range(3)] for _ in range(T)]
    for t in range(T):
        mem[t][0][0] = mem[t][1][0] = True
        mem[t][0][1] = True
        mem[t][1][2] = True
    go = [[False, False, False, True, True] for _ in range(T)]
    fr = (0, 1, 2)
    cases.append(dict(
        name="membership_anchor", P=5, N=3, L=4, KL=2, KG=3, n_frames=3, n_block=3,
        local_attn=-1, agent=(fr,) * 5, local=(fr,) * 3, glob=fr,
        local_active=((True,) * 3, (True,) * 3, (False,) * 3),
        labels=None, q_active=((True, True, False),) * 3, direct=True, block_m=4,
        membership=mem, global_only=go, no_local=False))
    # No-local topology.
    fr = (2, 3, 4, 5)
    cases.append(dict(
        name="nolocal", P=3, N=2, L=4, KL=0, KG=3, n_frames=2, n_block=2, local_attn=4,
        agent=(fr,) * 3, local=(), glob=fr, local_active=(), labels=((0, 0, 1),) * 2,
        q_active=((True, True),) * 2, direct=True, block_m=4, membership=None,
        global_only=None, no_local=True))
    return cases


def gen_segmented(out: dict):
    import torch
    from multics.models.kernels.hier_segmented_attention import _build_metadata
    from multics.models.kernels.hier_packed_attention import _get_varlen_plan

    names = []
    for c in _seg_cases():
        for bm_kind in ("tile", "segment"):
            block_m = c["block_m"] if bm_kind == "tile" else max(c["L"], c["KL"], c["KG"], 1)
            res = _build_metadata(
                device="cpu", P=c["P"], N=c["N"], L=c["L"], KL=c["KL"], KG=c["KG"],
                n_frames=c["n_frames"], n_block=c["n_block"], local_attn=c["local_attn"],
                agent_frame_lists=c["agent"], local_frame_lists=c["local"],
                global_frame_list=c["glob"], local_active_frames=c["local_active"],
                labels=c["labels"], q_active=c["q_active"], direct_player=c["direct"],
                block_m=block_m, membership=c["membership"], global_only=c["global_only"],
                hier_no_local_hub=c["no_local"],
            )
            nm = f"{c['name']}/{bm_kind}"
            names.append(nm)
            meta = {k: c[k] for k in ("P", "N", "L", "KL", "KG", "n_frames", "n_block",
                                      "local_attn", "direct", "no_local")}
            meta["block_m"] = block_m
            meta["agent"] = [list(x) for x in c["agent"]]
            meta["local"] = [list(x) for x in c["local"]]
            meta["glob"] = list(c["glob"])
            meta["local_active"] = [list(x) for x in c["local_active"]]
            meta["labels"] = None if c["labels"] is None else [list(x) for x in c["labels"]]
            meta["q_active"] = [list(x) for x in c["q_active"]]
            meta["membership"] = c["membership"]
            meta["global_only"] = c["global_only"]
            out[f"{nm}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
            for key, val in zip(("prog_qbase", "prog_nq", "prog_seg", "kv_index", "kv_count"),
                                res[:5]):
                out[f"{nm}/{key}"] = val.numpy().astype(np.int32)
            out[f"{nm}/logical_pairs"] = np.array(int(res[5]), dtype=np.int64)
            if bm_kind == "segment":
                S = (c["P"] * c["n_frames"] * c["L"]
                     + c["n_frames"] * (c["N"] * c["KL"] + c["KG"]))
                plan = _get_varlen_plan(kv_index=res[3], kv_count=res[4], qbase=res[0],
                                        qlen=res[1], seg_ids=res[2], query_tokens=S)
                for key in ("q_index", "k_index", "cu_q", "cu_k"):
                    out[f"{nm}/plan_{key}"] = plan[key].numpy().astype(np.int64)
                out[f"{nm}/plan_scalars"] = np.array(
                    [plan["max_q"], plan["max_k"], plan["min_k_index"], plan["max_k_index"]],
                    dtype=np.int64)
    out["seg_case_names"] = np.frombuffer(json.dumps(names).encode(), dtype=np.uint8)
    del torch


# ---------------------------------------------------------------------------
# tiled layouts
# ---------------------------------------------------------------------------


def gen_tiled(out: dict):
    import torch
    from multics.models.kernels.hier_tiled_attention import (
        build_hier_tiled_cached_layout,
        build_hier_tiled_full_sequence_layouts,
        clear_hier_tiled_layout_cache,
    )

    names = []

    def save(nm, layouts, meta):
        names.append(nm)
        out[f"{nm}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        out[f"{nm}/n_layouts"] = np.array(len(layouts), dtype=np.int64)
        for i, lay in enumerate(layouts):
            for key in ("prog_qbase", "prog_nq", "prog_seg", "kv_index", "kv_count"):
                out[f"{nm}/{i}/{key}"] = getattr(lay, key).numpy().astype(np.int32)
            out[f"{nm}/{i}/kv_valid"] = lay.kv_valid.numpy().astype(np.uint8)
            out[f"{nm}/{i}/slots"] = np.array(
                [lay.logical_slots, lay.physical_slots, lay.dense_slots], dtype=np.int64)

    clear_hier_tiled_layout_cache()
    full_cases = []
    lab9 = torch.tensor(
        [[0, 0, 1, 1]] * 3 + [[0, 2, 2, 0]] * 3 + [[1, 1, 2, 2]] * 3, dtype=torch.long)
    act9 = torch.zeros(9, 3, dtype=torch.bool)
    act9.scatter_(1, lab9, True)
    for direct in (False, True):
        full_cases.append((f"full_refA_d{int(direct)}", 4, 9, 7, 3, 2, 3, 3, 4, lab9, act9,
                           direct))
    labB = torch.tensor([[0, 0, 1, 1]] * 3 + [[0, 1, 0, 1]] * 3 + [[1, 1, 0, 0]] * 3)
    full_cases.append(("full_refB", 4, 9, 5, 2, 2, 3, 3, 4, labB,
                       torch.ones(9, 2, dtype=torch.bool), True))
    act_off = act9.clone()
    act_off[3:6, 1] = False
    full_cases.append(("full_inactive", 4, 9, 7, 3, 2, 3, 3, -1, lab9, act_off, True))
    for nm, P, T, L, N, KL, KG, n, win, lab, act, direct in full_cases:
        clear_hier_tiled_layout_cache()
        lays = build_hier_tiled_full_sequence_layouts(
            device=torch.device("cpu"), num_players=P, num_frames=T, num_patches=L,
            num_groups=N, num_local_hub_tokens=KL, num_global_hub_tokens=KG,
            num_frame_per_block=n, local_attn_size=win, group_labels=lab,
            active_group=act, direct_player=direct)
        meta = dict(P=P, T=T, L=L, N=N, KL=KL, KG=KG, n=n, win=win, direct=direct,
                    labels=lab.tolist(), active=act.tolist())
        save(nm, lays, meta)
    # Cached layouts (tests/test_hier_tiled_layout.py:301-358) for every block.
    P, T, L, N, KL, KG, n, window = 4, 9, 5, 2, 2, 3, 3, 4
    retention = window + n
    act = torch.ones(T, N, dtype=torch.bool)
    act[4, 1] = False
    for bi, bs in enumerate(range(0, T, n)):
        be = bs + n
        retained = tuple(range(max(0, be - retention), be))
        clear_hier_tiled_layout_cache()
        lab_rows = tuple(tuple(int(x) for x in r) for r in labB[bs:be].tolist())
        q_act = tuple(tuple(bool(x) for x in r) for r in act[bs:be].tolist())
        la = tuple(tuple(bool(act[f, g]) for f in retained) for g in range(N))
        for direct in (False, True):
            lay = build_hier_tiled_cached_layout(
                device=torch.device("cpu"), P=P, N=N, L=L, KL=KL, KG=KG, n_frames=n,
                n_block=n, local_attn=window, agent_frame_lists=(retained,) * P,
                local_frame_lists=(retained,) * N, global_frame_list=retained,
                local_active_frames=la, labels=lab_rows, q_active=q_act,
                direct_player=direct)
            meta = dict(P=P, N=N, L=L, KL=KL, KG=KG, n_frames=n, n_block=n,
                        local_attn=window, agent=[list(retained)] * P,
                        local=[list(retained)] * N, glob=list(retained),
                        local_active=[list(x) for x in la],
                        labels=[list(x) for x in lab_rows],
                        q_active=[list(x) for x in q_act], direct=direct)
            save(f"cached_b{bi}_d{int(direct)}", (lay,), meta)
    out["tiled_case_names"] = np.frombuffer(json.dumps(names).encode(), dtype=np.uint8)


# ---------------------------------------------------------------------------
# numerics
# ---------------------------------------------------------------------------


def _bf16_round(t):
    import torch

    return t.to(torch.bfloat16).to(torch.float32)


def _bf16_bits(t):
    import torch

    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def gen_numerics(out: dict, attn_mod):
    import torch
    from multics.data.dataset import _camera12_from_absolute_c2w
    from multics.models.hier_masks import build_stage2_hier_self_attn_mask
    from multics.models.rope import (
        build_hub_freqs_4d,
        build_multiplayer_freqs_4d,
        build_simplex_vertices,
        precompute_freqs_cis_4d_wan_rerope,
        rope_apply,
    )

    cases = [
        # name, H, D, splits, pool, labels-mode flags
        ("cfg1_d64", 4, 64, (6, 16, 20, 22), 8, dict(n=1, win=-1, membership=False)),
        ("cfg1_d128", 2, 128, (12, 32, 42, 42), 10, dict(n=1, win=-1, membership=False)),
        ("cfg1_d128_n3", 2, 128, (12, 32, 42, 42), 10, dict(n=3, win=21, membership=False)),
        ("cfg1_d128_mem", 2, 128, (12, 32, 42, 42), 10, dict(n=1, win=-1, membership=True)),
    ]
    P, T, h, w, N, KL, KG = 4, 3, 4, 4, 2, 8, 6
    L = h * w
    S = P * T * L + T * (N * KL + KG)
    names = []
    for name, H, D, splits, pool, flags in cases:
        g = torch.Generator().manual_seed(0)
        dim = H * D
        qx = _bf16_round(torch.randn(1, S, dim, generator=g))
        kx = _bf16_round(torch.randn(1, S, dim, generator=g))
        v = _bf16_round(torch.randn(1, S, dim, generator=g))
        # Per-player per-frame random SE(3) poses -> camera12.
        ang = (torch.rand(P, T, 3, generator=g, dtype=torch.float64) * 2 - 1) * math.pi
        trans = torch.randn(P, T, 3, generator=g, dtype=torch.float64)
        c2w = torch.zeros(P, T, 4, 4, dtype=torch.float64)
        c2w[..., :3, :3] = _euler_zyx(ang)
        c2w[..., :3, 3] = trans
        c2w[..., 3, 3] = 1.0
        cam12 = _camera12_from_absolute_c2w(c2w, pos_scale=1.0)  # [P,T,12]
        cam = torch.zeros(1, S, 12)
        cam[0, : P * T * L] = cam12[:, :, None, :].expand(P, T, L, 12).reshape(-1, 12)
        cam = _bf16_round(cam)
        wcq = _bf16_round(torch.randn(dim, 12, generator=g) * 0.02)
        wck = _bf16_round(torch.randn(dim, 12, generator=g) * 0.02)
        nqw = _bf16_round(1 + torch.randn(dim, generator=g) * 0.02)
        nkw = _bf16_round(1 + torch.randn(dim, generator=g) * 0.02)
        # Freqs exactly as WanModel.build_self_attn_freqs_with_hub builds them
        # (wan_video_dit.py:338-359): simplex 4D player freqs ++ hub freqs.
        bands = precompute_freqs_cis_4d_wan_rerope(D, splits=splits)
        verts = build_simplex_vertices(pool, splits[1])
        agent_f = build_multiplayer_freqs_4d(bands, T, h, w, list(range(P)), verts, 1.0,
                                             device=torch.device("cpu"))
        hub_f = build_hub_freqs_4d(bands, T, N * KL + KG, device=torch.device("cpu"))
        freqs = torch.cat([agent_f, hub_f], dim=0)
        if flags["membership"]:
            mem = torch.zeros(T, N, P, dtype=torch.bool)
            mem[:, 0, 0] = mem[:, 0, 1] = True
            mem[:, 1, 1] = mem[:, 1, 2] = True
            go = torch.zeros(T, P, dtype=torch.bool)
            go[:, 3] = True
            labels = torch.zeros(T, P, dtype=torch.long)
            mask = build_stage2_hier_self_attn_mask(
                P, T, L, N, KL, KG, flags["n"], flags["win"], labels, None, True,
                torch.device("cpu"), membership=mem, global_only=go)
        else:
            mem = go = None
            labels = torch.tensor([[0, 0, 1, 1]] * T)
            mask = build_stage2_hier_self_attn_mask(
                P, T, L, N, KL, KG, flags["n"], flags["win"], labels, None, True,
                torch.device("cpu"))
        layer = attn_mod.SelfAttention(dim, H, eps=1e-6).float().eval()
        layer.enable_camera_pose_qk(12, dropout_p=0.0)
        with torch.no_grad():
            layer.cam_q.weight.copy_(wcq)
            layer.cam_k.weight.copy_(wck)
            layer.norm_q.weight.copy_(nqw)
            layer.norm_k.weight.copy_(nkw)
            qc, kc = layer._apply_camera_qk(qx, kx, cam)
            qn = layer.norm_q(qc)
            kn = layer.norm_k(kc)
            q = rope_apply(qn, freqs, H)
            k = rope_apply(kn, freqs, H)
            o = attn_mod.flash_attention(q, k, v, num_heads=H, mask=mask)
        names.append(name)
        meta = dict(P=P, T=T, h=h, w=w, L=L, N=N, KL=KL, KG=KG, H=H, D=D, S=S,
                    n=flags["n"], win=flags["win"], membership=flags["membership"],
                    direct=True, splits=list(splits), pool=pool)
        out[f"{name}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        out[f"{name}/qx"] = _bf16_bits(qx[0])
        out[f"{name}/kx"] = _bf16_bits(kx[0])
        out[f"{name}/v"] = _bf16_bits(v[0])
        out[f"{name}/cam"] = _bf16_bits(cam[0])
        out[f"{name}/wcq"] = _bf16_bits(wcq)
        out[f"{name}/wck"] = _bf16_bits(wck)
        out[f"{name}/nqw"] = _bf16_bits(nqw)
        out[f"{name}/nkw"] = _bf16_bits(nkw)
        out[f"{name}/freqs"] = torch.view_as_real(freqs[:, 0]).numpy().astype(np.float64)
        out[f"{name}/cam12"] = cam12.numpy().astype(np.float32)
        out[f"{name}/labels"] = labels.numpy().astype(np.int64)
        if mem is not None:
            out[f"{name}/membership"] = mem.numpy()
            out[f"{name}/global_only"] = go.numpy()
        out[f"{name}/roped_q"] = q[0].numpy().astype(np.float32)
        out[f"{name}/roped_k"] = k[0].numpy().astype(np.float32)
        out[f"{name}/out"] = o[0].numpy().astype(np.float32)
        out[f"{name}/mask_popcount"] = np.array(int(mask.sum()), dtype=np.int64)
    out["num_case_names"] = np.frombuffer(json.dumps(names).encode(), dtype=np.uint8)


def gen_action(out: dict, attn_mod):
    import torch
    from einops import repeat
    from multics.models.hier_masks import get_temporal_block_causal_mask
    from multics.models.rope import precompute_freqs_cis

    mask_cases = [(42, 1, -1), (42, 7, 24), (21, 3, 21), (9, 7, 24), (5, 2, 3), (12, 4, 6)]
    for F, n, win in mask_cases:
        out[f"temporal/{F}_{n}_{win}"] = get_temporal_block_causal_mask(F, n, win).numpy()
    kb_cases = [(6, 3, -1, 5), (9, 3, 4, 7)]
    for F, n, win, L in kb_cases:
        fm = get_temporal_block_causal_mask(F, n, win)
        out[f"keyboard/{F}_{n}_{win}_{L}"] = repeat(fm, "f g -> (f q) (g k)", q=L, k=12).numpy()
    out["mask_cases"] = np.array(mask_cases, dtype=np.int64)
    out["kb_cases"] = np.array(kb_cases, dtype=np.int64)

    H, D = 2, 128
    dim = H * D
    g = torch.Generator().manual_seed(0)

    def lin_params(prefix, layer):
        with torch.no_grad():
            layer.weight.copy_(_bf16_round(torch.randn(layer.weight.shape, generator=g) * 0.05))
            if layer.bias is not None:
                layer.bias.copy_(_bf16_round(torch.randn(layer.bias.shape, generator=g) * 0.05))
        out[f"{prefix}.weight"] = _bf16_bits(layer.weight.detach())
        if layer.bias is not None:
            out[f"{prefix}.bias"] = _bf16_bits(layer.bias.detach())

    def norm_params(prefix, norm):
        with torch.no_grad():
            norm.weight.copy_(_bf16_round(1 + torch.randn(norm.weight.shape, generator=g) * 0.02))
        out[f"{prefix}.weight"] = _bf16_bits(norm.weight.detach())

    # per-frame action attention: SelfAttention over [B, F, dim] with 1-D RoPE
    B, F, n, win = 7, 9, 3, 4
    sa = attn_mod.SelfAttention(dim, H, eps=1e-6).float().eval()
    for name in ("q", "k", "v", "o"):
        lin_params(f"temporal/{name}", getattr(sa, name))
    norm_params("temporal/norm_q", sa.norm_q)
    norm_params("temporal/norm_k", sa.norm_k)
    x = _bf16_round(torch.randn(B, F, dim, generator=g))
    freqs = precompute_freqs_cis(D, end=F).unsqueeze(1)
    mask = get_temporal_block_causal_mask(F, n, win)
    with torch.no_grad():
        y = sa(x, freqs, mask)
    out["temporal/x"] = _bf16_bits(x)
    out["temporal/out"] = y.numpy().astype(np.float32)
    out["temporal/shape"] = np.array([B, F, n, win, H, D], dtype=np.int64)

    # keyboard cross-attention: CrossAttention under the repeated frame mask
    P, F, n, win, L, K = 2, 6, 2, -1, 5, 12
    ca = attn_mod.CrossAttention(dim, H, eps=1e-6).float().eval()
    for name in ("q", "k", "v", "o"):
        lin_params(f"keyboard/{name}", getattr(ca, name))
    norm_params("keyboard/norm_q", ca.norm_q)
    norm_params("keyboard/norm_k", ca.norm_k)
    xq = _bf16_round(torch.randn(P, F * L, dim, generator=g))
    ctx = _bf16_round(torch.randn(P, F * K, dim, generator=g))
    kmask = repeat(get_temporal_block_causal_mask(F, n, win), "f g -> (f q) (g k)", q=L, k=K)
    with torch.no_grad():
        y = ca(xq, ctx, kmask)
    out["keyboard/x"] = _bf16_bits(xq)
    out["keyboard/ctx"] = _bf16_bits(ctx)
    out["keyboard/out"] = y.numpy().astype(np.float32)
    out["keyboard/shape"] = np.array([P, F, n, win, L, K, H, D], dtype=np.int64)


def gen_grads(out: dict, attn_mod):
    """Reads the inputs recorded in numerics.npz (run it first)."""
    import torch
    from multics.models.hier_masks import build_stage2_hier_self_attn_mask
    from multics.models.rope import rope_apply

    num = np.load(HERE / "numerics.npz")

    def bf(a):
        return torch.from_numpy(a.astype(np.uint16).view(np.int16)).view(torch.bfloat16).float()

    names = []
    for name in ("cfg1_d128", "cfg1_d128_n3", "cfg1_d128_mem"):
        meta = json.loads(bytes(num[f"{name}/meta"]).decode())
        H, S = meta["H"], meta["S"]
        qx, kx, v = (bf(num[f"{name}/{t}"])[None].requires_grad_(True) for t in ("qx", "kx", "v"))
        cam = bf(num[f"{name}/cam"])[None]
        wcq, wck, nqw, nkw = (bf(num[f"{name}/{t}"]) for t in ("wcq", "wck", "nqw", "nkw"))
        fr = torch.from_numpy(num[f"{name}/freqs"])
        freqs = torch.complex(fr[..., 0], fr[..., 1]).unsqueeze(1)
        P, T, L, N, KL, KG = (meta[k] for k in ("P", "T", "L", "N", "KL", "KG"))
        labels = torch.from_numpy(num[f"{name}/labels"])
        if meta["membership"]:
            mask = build_stage2_hier_self_attn_mask(
                P, T, L, N, KL, KG, meta["n"], meta["win"], labels, None, True,
                torch.device("cpu"), membership=torch.from_numpy(num[f"{name}/membership"]),
                global_only=torch.from_numpy(num[f"{name}/global_only"]))
        else:
            mask = build_stage2_hier_self_attn_mask(P, T, L, N, KL, KG, meta["n"], meta["win"],
                                                    labels, None, True, torch.device("cpu"))
        layer = attn_mod.SelfAttention(H * meta["D"], H, eps=1e-6).float()
        layer.enable_camera_pose_qk(12, dropout_p=0.0)
        with torch.no_grad():
            layer.cam_q.weight.copy_(wcq)
            layer.cam_k.weight.copy_(wck)
            layer.norm_q.weight.copy_(nqw)
            layer.norm_k.weight.copy_(nkw)
        qc, kc = layer._apply_camera_qk(qx, kx, cam)
        q = rope_apply(layer.norm_q(qc), freqs, H)
        k = rope_apply(layer.norm_k(kc), freqs, H)
        o = attn_mod.flash_attention(q, k, v, num_heads=H, mask=mask)
        g = torch.Generator().manual_seed(7)
        dout = _bf16_round(torch.randn(o.shape, generator=g))
        (o * dout).sum().backward()
        names.append(name)
        out[f"{name}/dout"] = _bf16_bits(dout[0])
        for t, grad in (("qx", qx.grad[0]), ("kx", kx.grad[0]), ("v", v.grad[0]),
                        ("wcq", layer.cam_q.weight.grad), ("wck", layer.cam_k.weight.grad),
                        ("nqw", layer.norm_q.weight.grad), ("nkw", layer.norm_k.weight.grad)):
            out[f"{name}/d_{t}"] = grad.detach().numpy().astype(np.float32)
    out["grad_case_names"] = np.frombuffer(json.dumps(names).encode(), dtype=np.uint8)


def _euler_zyx(ang):
    import torch

    z, y, x = ang[..., 0], ang[..., 1], ang[..., 2]
    cz, sz, cy, sy, cx, sx = z.cos(), z.sin(), y.cos(), y.sin(), x.cos(), x.sin()
    R = torch.zeros(*ang.shape[:-1], 3, 3, dtype=ang.dtype)
    R[..., 0, 0] = cz * cy
    R[..., 0, 1] = cz * sy * sx - sz * cx
    R[..., 0, 2] = cz * sy * cx + sz * sx
    R[..., 1, 0] = sz * cy
    R[..., 1, 1] = sz * sy * sx + cz * cx
    R[..., 1, 2] = sz * sy * cx - cz * sx
    R[..., 2, 0] = -sy
    R[..., 2, 1] = cy * sx
    R[..., 2, 2] = cy * cx
    return R


# ---------------------------------------------------------------------------
# cached (causal) forward of SelfAttention over consecutive blocks
# ---------------------------------------------------------------------------


def _bits(t):
    import torch

    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().astype(np.uint16)


def _causal_cases():
    return [
        # tests/test_hier_segmented_causal_forward.py:58-127 shape: initial append,
        # steady state, regrouping between blocks, rolling eviction
        dict(name="labels_dyn", P=4, N=2, L=16, KL=3, KG=2, n=2, n_block=2, local_attn=4,
             heads=2, blocks=4, cam=False, membership=False, no_local=False),
        dict(name="cam_membership", P=4, N=2, L=12, KL=3, KG=2, n=2, n_block=2, local_attn=4,
             heads=2, blocks=4, cam=True, membership=True, no_local=False),
        dict(name="no_local", P=3, N=2, L=16, KL=0, KG=3, n=1, n_block=1, local_attn=3,
             heads=2, blocks=5, cam=False, membership=False, no_local=True),
    ]


def gen_causal(out: dict):
    """``SelfAttention.causal_forward_hier_hub`` (``multics/models/attention.py:456-1005``)
    with the SDPA backend, block after block over rolling caches
    (``_rolling_cache_append`` / ``_rolling_bool_cache_append``, ``:90-228``)."""
    import torch

    from multics.models.wan_video_dit import SelfAttention

    os.environ["WAN_HIER_INFER_KERNEL"] = "sdpa"
    names = []
    for c in _causal_cases():
        g = torch.Generator().manual_seed(17)
        P, N, L, KL, KG, n = c["P"], c["N"], c["L"], c["KL"], c["KG"], c["n"]
        H, D = c["heads"], 128
        dim = H * D
        retention = c["local_attn"] + n
        S = P * n * L + n * (N * KL + KG)
        torch.manual_seed(5)
        layer = SelfAttention(dim=dim, num_heads=H)
        if c["cam"]:
            layer.enable_camera_pose_qk(12, dropout_p=0.0)
        layer = layer.to(dtype=torch.bfloat16).eval()
        layer.num_frame_per_block = c["n_block"]
        layer.local_attn_size = c["local_attn"]
        if c["no_local"]:
            layer.hier_no_local_hub = True
        with torch.no_grad():
            for nrm in (layer.norm_q, layer.norm_k):
                nrm.weight.copy_(1 + 0.02 * torch.randn(dim, generator=g))
            if c["cam"]:
                layer.cam_q.weight.copy_(0.02 * torch.randn(dim, 12, generator=g))
                layer.cam_k.weight.copy_(0.02 * torch.randn(dim, 12, generator=g))

        def stream(cap):
            return {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16),
                    "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16),
                    "global_end_index": torch.zeros(1, dtype=torch.long),
                    "local_end_index": torch.zeros(1, dtype=torch.long)}

        cache = {"hier_hub": True, "sparse_hub": True, "num_players": P, "num_groups": N,
                 "num_local_hub_tokens": KL, "num_global_hub_tokens": KG,
                 "hier_no_local_hub": c["no_local"],
                 "agent_caches": [stream(retention * L) for _ in range(P)],
                 "local_hubs": [] if c["no_local"] else [stream(retention * KL) for _ in range(N)],
                 "global_hub": stream(retention * max(KG, 1))}
        for lc in cache["local_hubs"]:
            lc["active"] = torch.zeros(retention * KL, dtype=torch.bool)
        T_full = c["blocks"] * n
        mem = go = None
        if c["membership"]:
            mem = torch.zeros(T_full, N, P, dtype=torch.bool)
            mem[:, 0, 0] = mem[:, 0, 1] = True
            mem[:, 1, 2] = True
            mem[n:2 * n, 1, 1] = True  # player 1 anchors both groups in block 1
            go = torch.zeros(T_full, P, dtype=torch.bool)
            go[:, 3] = True
            out[f"{c['name']}/membership"] = mem.numpy().astype(np.uint8)
            out[f"{c['name']}/global_only"] = go.numpy().astype(np.uint8)
        nm = c["name"]
        for k_, v_ in layer.state_dict().items():
            # the q/k/v/o weights are the same seeded set for every case
            key = f"{nm}/w/{k_}" if (k_.startswith("cam_") or k_.startswith("norm_")) else f"w/{k_}"
            out[key] = _bits(v_)
        with torch.inference_mode():
            for blk in range(c["blocks"]):
                x = torch.randn(1, S, dim, generator=g).to(torch.bfloat16)
                phase = torch.rand(S, 1, D // 2, generator=g, dtype=torch.float64) * 2 * math.pi
                freqs = torch.polar(torch.ones_like(phase), phase)
                row = (0, 0, 1, 1)[:P] if blk % 2 == 0 else (0, 1, 0, 1, 1)[:P]
                labels = torch.tensor([row] * n, dtype=torch.long)
                active = torch.ones(n, N, dtype=torch.bool)
                cam = None
                if c["cam"]:
                    cam = torch.zeros(1, S, 12)
                    cam[0, : P * n * L] = torch.randn(P * n, 12, generator=g).repeat_interleave(L, 0)
                    cam = cam.to(torch.bfloat16)
                kw = dict(current_start=blk * n * P * L, num_frames=n, num_players=P,
                          num_hub_tokens=N * KL + KG, cam_tokens=cam, direct_player=True)
                if c["membership"]:
                    kw.update(membership=mem, global_only=go, active_group=None)
                else:
                    kw.update(group_labels=labels, active_group=active)
                y = layer.causal_forward_hier_hub(x, freqs, cache, **kw)
                out[f"{nm}/{blk}/x"] = _bits(x[0])
                out[f"{nm}/{blk}/freqs"] = np.stack([freqs[:, 0].real.numpy(),
                                                      freqs[:, 0].imag.numpy()],
                                                     -1).astype(np.float32)
                out[f"{nm}/{blk}/labels"] = labels.numpy()
                out[f"{nm}/{blk}/active"] = active.numpy().astype(np.uint8)
                if cam is not None:
                    out[f"{nm}/{blk}/cam"] = _bits(cam[0])
                out[f"{nm}/{blk}/out"] = _bits(y[0])
        streams = cache["agent_caches"] + cache["local_hubs"] + [cache["global_hub"]]
        for i, st in enumerate(streams):
            out[f"{nm}/cache/{i}/k"] = _bits(st["k"][0])
            out[f"{nm}/cache/{i}/v"] = _bits(st["v"][0])
            out[f"{nm}/cache/{i}/idx"] = np.array(
                [int(st["global_end_index"]), int(st["local_end_index"])], np.int64)
            if "active" in st:
                out[f"{nm}/cache/{i}/active"] = st["active"].numpy().astype(np.uint8)
        meta = {k_: v_ for k_, v_ in c.items()}
        meta["retention"] = retention
        meta["S"] = S
        meta["n_streams"] = len(streams)
        out[f"{nm}/meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        names.append(nm)
    out["causal_case_names"] = np.frombuffer(json.dumps(names).encode(), dtype=np.uint8)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default=None, help="write one fixture file (e.g. causal)")
    args = ap.parse_args()
    attn_mod = _setup(args.reference)
    import torch

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for fname, fn in (("masks", lambda o: gen_masks(args.reference, o)),
                      ("segmented", gen_segmented), ("tiled", gen_tiled),
                      ("numerics", lambda o: gen_numerics(o, attn_mod)),
                      ("action", lambda o: gen_action(o, attn_mod)),
                      ("grads", lambda o: gen_grads(o, attn_mod)),
                      ("causal", gen_causal)):
        if args.only and fname != args.only:
            continue
        out: dict = {}
        fn(out)
        path = HERE / f"{fname}.npz"
        np.savez_compressed(path, **out)
        print(f"wrote {path} ({path.stat().st_size / 1024:.1f} KiB, {len(out)} arrays)")


if __name__ == "__main__":
    main()

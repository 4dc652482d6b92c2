"""CPU oracle for the hierarchical group-attention hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and there only as the checker or as the timed CPU baseline.  The
product path (``multics_b200``) never imports it.

It restates in NumPy the reference algorithm of TencentARC/Multics for the
hierarchical attention path.  Each function cites the reference function it
follows (paths relative to the Multics checkout).  Parity of this restatement
is pinned against fixtures generated from the reference itself
(``tests/golden/gen_golden.py`` imports the reference and records its
outputs; ``tests/test_oracle_golden.py`` checks every function here against
them).

Token order everywhere (``multics/models/hier_masks.py:381,418-440``)::

    [P*T*L players (player-major, frame, patch) | T*N*KL local hubs (frame,
     group, slot) | T*KG global hubs (frame, slot)]
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np


# ---------------------------------------------------------------------------
# dense mask (hier_masks.py:364-641)
# ---------------------------------------------------------------------------


def token_ids(P, T, L, N, KL, KG, S_pad=None):
    """Per-token kind/time/player/group ids (``hier_masks.py:418-440``).

    With ``S_pad`` the arrays are padded like the Flex builder does
    (``hier_masks.py:784-805``): padded tokens are none of the three kinds.
    """
    A = P * T * L
    LS = T * N * KL
    S = A + LS + T * KG
    n = S if S_pad is None else S_pad
    idx = np.arange(n, dtype=np.int64)
    valid = idx < S
    is_player = valid & (idx < A)
    is_local = valid & (idx >= A) & (idx < A + LS)
    is_global = valid & (idx >= A + LS)
    t_id = np.zeros(n, np.int64)
    p_id = np.zeros(n, np.int64)
    g_id = np.zeros(n, np.int64)
    a = idx[is_player]
    p_id[is_player] = a // (T * L)
    t_id[is_player] = a % (T * L) // L
    if KL > 0:
        loc = idx[is_local] - A
        t_id[is_local] = loc // (N * KL)
        g_id[is_local] = loc % (N * KL) // KL
    if KG > 0:
        t_id[is_global] = (idx[is_global] - A - LS) // KG
    return dict(idx=idx, valid=valid, is_player=is_player, is_local=is_local,
                is_global=is_global, t=t_id, p=p_id, g=g_id, S=S)


def active_from_labels(labels, N):
    """``active.scatter_(1, labels, True)`` (``hier_masks.py:55-57``)."""
    labels = np.asarray(labels, np.int64)
    T = labels.shape[0]
    active = np.zeros((T, N), bool)
    for t in range(T):
        active[t, labels[t]] = True
    return active


def validate_labels(labels, T, P, N):
    """Shape/range checks of ``_prepare_hier_group_tensors`` (``hier_masks.py:44-54``)."""
    labels = np.asarray(labels)
    if labels.ndim == 3:
        if labels.shape[0] != 1:
            raise ValueError(f"hier_hub expects group_labels batch B=1, got {tuple(labels.shape)}")
        labels = labels[0]
    if labels.shape != (T, P):
        raise ValueError(f"group_labels must be [T={T},P={P}], got {tuple(labels.shape)}")
    if labels.size and (labels.min() < 0 or labels.max() >= N):
        raise ValueError(
            f"group_labels values must be in [0,{N}), got min={int(labels.min())} max={int(labels.max())}")
    return labels.astype(np.int64)


def unit_pred(qk, kk, qt, kt, qp, kp, qg, kg, *, n_block, local_attn, direct, no_local,
              labels=None, active=None, membership=None, global_only=None):
    """Elementwise hierarchical edge predicate.

    Arguments are broadcastable integer arrays: ``qk``/``kk`` are token kinds
    (0 player, 1 local, 2 global, 3 padding), ``qt``/``kt`` frames, ``qp``/``kp``
    players, ``qg``/``kg`` groups.  The eleven edge sets are those of
    ``build_stage2_hier_self_attn_mask`` (labels, ``hier_masks.py:453-507``) and
    of ``_build_stage2_hier_self_attn_mask_membership`` (``hier_masks.py:584-641``),
    except the token-level inactive-local self edge (``:484-486`` /
    ``:618-620``) which the callers add on the diagonal.
    """
    q_player, k_player = qk == 0, kk == 0
    q_local, k_local = qk == 1, kk == 1
    q_global, k_global = qk == 2, kk == 2
    q_block = qt // n_block
    k_block = kt // n_block
    m_window = k_block <= q_block
    if local_attn != -1:
        m_window = m_window & (qt - kt < local_attn)
    same_block = q_block == k_block
    T = active.shape[0]
    qtc = np.clip(qt, 0, T - 1)
    ktc = np.clip(kt, 0, T - 1)
    act_q = active[qtc, np.clip(qg, 0, active.shape[1] - 1)]
    act_k = active[ktc, np.clip(kg, 0, active.shape[1] - 1)]
    if membership is None:
        Pn = labels.shape[1]
        qpc = np.clip(qp, 0, Pn - 1)
        kpc = np.clip(kp, 0, Pn - 1)
        q_grp = labels[qtc, qpc]
        k_grp_at_qt = labels[qtc, kpc]
        same_group = q_grp == k_grp_at_qt
        q_in_kg = kg == q_grp
        k_in_qg = k_grp_at_qt == qg
        p2g = np.zeros_like(m_window)
        g2p = np.zeros_like(m_window)
    else:
        Pn = membership.shape[2]
        qpc = np.clip(qp, 0, Pn - 1)
        kpc = np.clip(kp, 0, Pn - 1)
        bits = (membership.astype(np.int64) << np.arange(membership.shape[1])[None, :, None]).sum(1)
        q_bits = bits[qtc, qpc]
        k_bits_at_qt = bits[qtc, kpc]
        same_group = (q_bits & k_bits_at_qt) != 0
        q_in_kg = ((q_bits >> np.clip(kg, 0, 62)) & 1) != 0
        k_in_qg = ((k_bits_at_qt >> np.clip(qg, 0, 62)) & 1) != 0
        q_go = global_only[qtc, qpc]
        k_go = global_only[ktc, kpc]
        p2g = q_player & k_global & q_go & m_window
        g2p = q_global & k_player & k_go & m_window
    if no_local:
        p2g = q_player & k_global & m_window
        g2p = q_global & k_player & m_window
    m = q_player & k_player & (qp == kp) & m_window
    if direct:
        m = m | (q_player & k_player & (qp != kp) & same_group & same_block)
    m = m | (q_player & k_local & act_k & q_in_kg & m_window)
    m = m | (q_local & act_q & k_player & k_in_qg & m_window)
    m = m | (q_local & act_q & k_global & m_window)
    m = m | (q_local & act_q & k_local & act_k & (qg == kg) & m_window)
    m = m | (q_global & k_local & act_k & m_window)
    m = m | (q_global & k_global & m_window)
    m = m | p2g | g2p
    return m


def _kinds(ids):
    k = np.full(ids["idx"].shape, 3, np.int64)
    k[ids["is_player"]] = 0
    k[ids["is_local"]] = 1
    k[ids["is_global"]] = 2
    return k


def prepare_grouping(P, T, N, labels=None, active=None, membership=None, global_only=None):
    """Normalise the grouping inputs like ``_prepare_hier_group_tensors`` /
    ``_prepare_hier_membership_tensors`` (``hier_masks.py:22-71,127-193``)."""
    if membership is not None:
        membership = np.asarray(membership, bool)
        if membership.ndim == 4:
            membership = membership[0]
        if global_only is None:
            raise ValueError("hier_group_format=membership requires global_only [T,P] or [1,T,P]")
        global_only = np.asarray(global_only, bool)
        if global_only.ndim == 3:
            global_only = global_only[0]
        if active is None:
            active = membership.any(-1)
        return None, np.asarray(active, bool), membership, global_only
    labels = validate_labels(labels, T, P, N)
    if active is None:
        active = active_from_labels(labels, N)
    return labels, np.asarray(active, bool), None, None


def dense_mask(P, T, L, N, KL, KG, n_block, local_attn, labels=None, active=None,
               direct=False, membership=None, global_only=None, no_local=False,
               rows: Optional[slice] = None):
    """Dense ``[S,S]`` bool mask (``build_stage2_hier_self_attn_mask``,
    ``hier_masks.py:364-641``).  ``rows`` restricts the output to a row range."""
    if no_local and (KL != 0 or KG <= 0):
        raise ValueError(f"hier_no_local_hub requires K_L=0 and K_G>0; got K_L={KL}, K_G={KG}")
    if local_attn != -1 and local_attn < n_block:
        raise ValueError(
            f"hier_hub requires local_attn_size=-1 or >= num_frame_per_block; got local_attn_size={local_attn}, n={n_block}")
    labels, active, membership, global_only = prepare_grouping(
        P, T, N, labels, active, membership, global_only)
    ids = token_ids(P, T, L, N, KL, KG)
    kinds = _kinds(ids)
    r = slice(None) if rows is None else rows
    q = lambda a: a[r][:, None]  # noqa: E731
    k = lambda a: a[None, :]  # noqa: E731
    m = unit_pred(q(kinds), k(kinds), q(ids["t"]), k(ids["t"]), q(ids["p"]), k(ids["p"]),
                  q(ids["g"]), k(ids["g"]), n_block=n_block, local_attn=local_attn,
                  direct=direct, no_local=no_local, labels=labels, active=active,
                  membership=membership, global_only=global_only)
    if KL > 0:
        qi = ids["idx"][r]
        qloc = ids["is_local"][r]
        inactive = qloc & ~active[ids["t"][r], ids["g"][r]]
        rr = np.nonzero(inactive)[0]
        m[rr, qi[rr]] = True
    return m


# ---------------------------------------------------------------------------
# Flex BlockMask (hier_masks.py:722-1149 + create_block_mask semantics)
# ---------------------------------------------------------------------------


def flex_block_lists(mask: np.ndarray, S_pad: int, block: int = 128):
    """Block-level reduction of a mask padded to ``S_pad``, as ``create_block_mask``
    does for the reference's ``mask_mod`` (padded rows/cols are masked,
    ``hier_masks.py:904``): returns ``(kv_num_blocks, kv_indices, full_num,
    full_indices)`` with partial and full block lists in ascending order."""
    S = mask.shape[0]
    nb = S_pad // block
    pad = np.zeros((S_pad, S_pad), bool)
    pad[:S, :S] = mask
    blk = pad.reshape(nb, block, nb, block).transpose(0, 2, 1, 3).reshape(nb, nb, -1)
    anyb = blk.any(-1)
    allb = blk.all(-1)
    partial = anyb & ~allb
    kvn = partial.sum(1).astype(np.int32)
    fn = allb.sum(1).astype(np.int32)
    kvi = np.concatenate([np.nonzero(partial[i])[0] for i in range(nb)]).astype(np.int32)
    fi = np.concatenate([np.nonzero(allb[i])[0] for i in range(nb)]).astype(np.int32)
    return kvn, kvi, fn, fi


def logical_pairs(P, T, L, N, KL, KG, n_block, local_attn, **kw):
    """Unmasked pair count (dense-mask popcount) computed row-chunk by row-chunk."""
    S = P * T * L + T * (N * KL + KG)
    total = 0
    step = max(1, int(2e7 // max(S, 1)))
    for r0 in range(0, S, step):
        total += int(dense_mask(P, T, L, N, KL, KG, n_block, local_attn,
                                rows=slice(r0, min(S, r0 + step)), **kw).sum())
    return total


def logical_pairs_units(P, T, L, N, KL, KG, n_block, local_attn, **kw):
    """The same count from the mask at unit scale (one token per player frame,
    local hub and global hub; L = K_L = K_G = 1), each unit pair weighted by
    its unit sizes.  The mask is uniform inside a unit pair except for an
    inactive local hub's self edge (``hier_masks.py:476-480``), a diagonal of
    K_L tokens rather than K_L x K_L."""
    if KL == 0 and KG == 0:
        return logical_pairs(P, T, L, N, KL, KG, n_block, local_attn, **kw)
    unit = dense_mask(P, T, 1, N, 1 if KL else 0, 1 if KG else 0, n_block, local_attn, **kw)
    sizes = np.concatenate([np.full(P * T, L), np.full(T * N if KL else 0, KL),
                            np.full(T if KG else 0, KG)]).astype(np.int64)
    w = sizes[:, None] * sizes[None, :]
    total = int((unit * w).sum())
    labels, active, _, _ = prepare_grouping(P, T, N, kw.get("labels"), kw.get("active"),
                                            kw.get("membership"), kw.get("global_only"))
    if KL:
        for t in range(T):
            for g in range(N):
                if not active[t, g]:
                    u = P * T + t * N + g
                    if unit[u, u]:
                        total -= KL * KL - KL
    return total


# ---------------------------------------------------------------------------
# segmented metadata (kernels/hier_segmented_attention.py:117-395)
# ---------------------------------------------------------------------------


def _temporal(qf, kf, n_block, local_attn):
    """``hier_segmented_attention.py:117-122``."""
    ok = (kf // n_block) <= (qf // n_block)
    if local_attn != -1:
        ok = ok and (qf - kf) < local_attn
    return ok


def segment_key_lists(*, P, N, L, KL, KG, n_frames, n_block, local_attn, agent, local, glob,
                      local_active, labels, q_active, direct, membership=None,
                      global_only=None, no_local=False):
    """Per-segment ``(qstart, qlen, [pool indices])`` of ``_build_metadata``
    (``hier_segmented_attention.py:247-368``).

    Pool order: agents ``(p*fa+fi)*L``, locals ``P*fa*L+(g*fl+fi)*KL``, globals
    after (``:247-258``).  Segment order: player-major agent rows, then
    frame-major (frame, group) local rows, then global rows.
    """
    fa = len(agent[0])
    fl = 0 if no_local else len(local[0])
    use_mem = membership is not None
    local_base = P * fa * L
    global_base = local_base + N * fl * KL
    A = lambda p, fi: list(range((p * fa + fi) * L, (p * fa + fi) * L + L))  # noqa: E731
    Lo = lambda g, fi: list(range(local_base + (g * fl + fi) * KL,  # noqa: E731
                                  local_base + (g * fl + fi) * KL + KL))
    G = lambda fi: list(range(global_base + fi * KG, global_base + fi * KG + KG))  # noqa: E731
    q_frames = tuple(glob[-n_frames:]) if KG > 0 else ()
    if len(q_frames) != n_frames:
        q_frames = tuple(agent[0][-n_frames:])
    segs = []
    for p in range(P):
        for qrel, qf in enumerate(q_frames):
            sel = []
            for fi, kf in enumerate(agent[p]):
                if _temporal(qf, kf, n_block, local_attn):
                    sel += A(p, fi)
            if direct:
                for o in range(P):
                    if o == p:
                        continue
                    if use_mem:
                        share = any(membership[qf][g][p] and membership[qf][g][o] for g in range(N))
                    else:
                        share = labels[qrel][o] == labels[qrel][p]
                    if not share:
                        continue
                    for fi, kf in enumerate(agent[o]):
                        if kf in q_frames and kf // n_block == qf // n_block:
                            sel += A(o, fi)
            if not no_local:
                owned = ([g for g in range(N) if membership[qf][g][p]] if use_mem
                         else [labels[qrel][p]])
                for g in owned:
                    for fi, kf in enumerate(local[g]):
                        if local_active[g][fi] and _temporal(qf, kf, n_block, local_attn):
                            sel += Lo(g, fi)
            if KG > 0 and (no_local or (use_mem and global_only[qf][p])):
                for fi, kf in enumerate(glob):
                    if _temporal(qf, kf, n_block, local_attn):
                        sel += G(fi)
            segs.append((p * n_frames * L + qrel * L, L, sel))
    aq = P * n_frames * L
    lq = n_frames * N * KL
    if not no_local:
        for qrel, qf in enumerate(q_frames):
            for g in range(N):
                sel = []
                if q_active[qrel][g]:
                    for p in range(P):
                        inside = membership[qf][g][p] if use_mem else labels[qrel][p] == g
                        if inside:
                            for fi, kf in enumerate(agent[p]):
                                if _temporal(qf, kf, n_block, local_attn):
                                    sel += A(p, fi)
                    for fi, kf in enumerate(local[g]):
                        if local_active[g][fi] and _temporal(qf, kf, n_block, local_attn):
                            sel += Lo(g, fi)
                    for fi, kf in enumerate(glob):
                        if _temporal(qf, kf, n_block, local_attn):
                            sel += G(fi)
                segs.append((aq + qrel * N * KL + g * KL, KL, sel))
    for qrel, qf in enumerate(q_frames):
        sel = []
        if not no_local:
            for g in range(N):
                for fi, kf in enumerate(local[g]):
                    if local_active[g][fi] and _temporal(qf, kf, n_block, local_attn):
                        sel += Lo(g, fi)
        for fi, kf in enumerate(glob):
            if _temporal(qf, kf, n_block, local_attn):
                sel += G(fi)
        if no_local:
            for p in range(P):
                for fi, kf in enumerate(agent[p]):
                    if _temporal(qf, kf, n_block, local_attn):
                        sel += A(p, fi)
        elif use_mem:
            for p in range(P):
                for fi, kf in enumerate(agent[p]):
                    if global_only[kf][p] and _temporal(qf, kf, n_block, local_attn):
                        sel += A(p, fi)
        segs.append((aq + lq + qrel * KG, KG, sel))
    return segs


def segmented_metadata(block_m, **kw):
    """``(prog_qbase, prog_nq, prog_seg, kv_index, kv_count, logical_pairs)`` of
    ``_build_metadata`` (``hier_segmented_attention.py:370-395``)."""
    segs = segment_key_lists(**kw)
    max_k = max(max((len(s[2]) for s in segs), default=1), 1)
    max_k = math.ceil(max_k / 64) * 64
    kv_index = np.zeros((len(segs), max_k), np.int32)
    kv_count = np.zeros(len(segs), np.int32)
    qb, qn, qs = [], [], []
    pairs = 0
    for sid, (q0, ql, sel) in enumerate(segs):
        kv_index[sid, : len(sel)] = sel
        kv_count[sid] = len(sel)
        pairs += ql * len(sel)
        for off in range(0, ql, block_m):
            qb.append(q0 + off)
            qn.append(min(block_m, ql - off))
            qs.append(sid)
    return (np.array(qb, np.int32), np.array(qn, np.int32), np.array(qs, np.int32),
            kv_index, kv_count, pairs)


def varlen_plan(prog_qbase, prog_nq, prog_seg, kv_index, kv_count, query_tokens):
    """``_get_varlen_plan`` (``kernels/hier_packed_attention.py:32-102``)."""
    qb = [int(x) for x in prog_qbase]
    qn = [int(x) for x in prog_nq]
    si = [int(x) for x in prog_seg]
    nk = [int(x) for x in kv_count]
    if si != list(range(len(si))):
        raise AssertionError("packed metadata must contain exactly one program per segment")
    cover = [r for b, n in zip(qb, qn) for r in range(b, b + n)]
    if cover != list(range(query_tokens)):
        raise AssertionError("packed query segments must partition the query sequence exactly")
    act = [s for s in si if qn[s] > 0 and nk[s] > 0]
    q_index = np.concatenate([np.arange(qb[s], qb[s] + qn[s]) for s in act]) if act else np.zeros(0, np.int64)
    k_index = np.concatenate([np.asarray(kv_index[s, : nk[s]], np.int64) for s in act]) if act else np.zeros(0, np.int64)
    cu_q = np.cumsum([0] + [qn[s] for s in act]).astype(np.int64)
    cu_k = np.cumsum([0] + [nk[s] for s in act]).astype(np.int64)
    return dict(q_index=q_index.astype(np.int64), k_index=k_index.astype(np.int64), cu_q=cu_q,
                cu_k=cu_k, max_q=max((qn[s] for s in act), default=0),
                max_k=max((nk[s] for s in act), default=0),
                min_k_index=int(k_index.min()) if k_index.size else 0,
                max_k_index=int(k_index.max()) if k_index.size else -1)


# ---------------------------------------------------------------------------
# tiled layouts (kernels/hier_tiled_attention.py:182-655)
# ---------------------------------------------------------------------------

TILED_BLOCK_M = 16
TILED_BLOCK_N = 128


@dataclass
class TiledLayout:
    prog_qbase: np.ndarray
    prog_nq: np.ndarray
    prog_seg: np.ndarray
    kv_index: np.ndarray
    kv_valid: np.ndarray
    kv_count: np.ndarray
    logical_slots: int
    physical_slots: int
    dense_slots: int


def pack_layout(dense_segments: Sequence[Sequence[tuple]], query_specs: Sequence[tuple]):
    """``_pack_layout`` (``hier_tiled_attention.py:182-241``)."""
    sel_segs = []
    logical = physical = dense_n = 0
    for dense in dense_segments:
        dense = list(dense)
        dense_n += len(dense)
        logical += sum(int(v) for _, v in dense)
        sel = []
        for s in range(0, len(dense), TILED_BLOCK_N):
            chunk = dense[s: s + TILED_BLOCK_N]
            if not any(v for _, v in chunk):
                continue
            chunk = chunk + [(0, False)] * (TILED_BLOCK_N - len(chunk))
            sel.extend(chunk)
        physical += len(sel)
        sel_segs.append(sel)
    max_k = max(max((len(x) for x in sel_segs), default=1), 1)
    max_k = math.ceil(max_k / TILED_BLOCK_N) * TILED_BLOCK_N
    kv_index = np.zeros((len(sel_segs), max_k), np.int32)
    kv_valid = np.zeros((len(sel_segs), max_k), np.uint8)
    kv_count = np.zeros(len(sel_segs), np.int32)
    qb, qn, qs = [], [], []
    for sid, ((q0, ql), sel) in enumerate(zip(query_specs, sel_segs)):
        if sel:
            kv_index[sid, : len(sel)] = [i for i, _ in sel]
            kv_valid[sid, : len(sel)] = [v for _, v in sel]
        kv_count[sid] = len(sel)
        for off in range(0, ql, TILED_BLOCK_M):
            qb.append(q0 + off)
            qn.append(min(TILED_BLOCK_M, ql - off))
            qs.append(sid)
    return TiledLayout(np.array(qb, np.int32), np.array(qn, np.int32), np.array(qs, np.int32),
                       kv_index, kv_valid, kv_count, logical, physical, dense_n)


def tiled_full_sequence_layouts(P, T, L, N, KL, KG, n, window, labels, active, direct):
    """``build_hier_tiled_full_sequence_layouts`` (``hier_tiled_attention.py:244-429``)."""
    labels = np.asarray(labels).tolist()
    active = np.asarray(active, bool).tolist()
    A = P * T * L
    gs = A + T * N * KL
    retention = T if window == -1 else window + n
    ab = lambda p, f: (p * T + f) * L  # noqa: E731
    lb = lambda g, f: A + (f * N + g) * KL  # noqa: E731
    gb = lambda f: gs + f * KG  # noqa: E731

    def app(d, base, width, ok):
        d.extend((base + t, bool(ok)) for t in range(width))

    out = []
    for bs in range(0, T, n):
        be = bs + n
        ret = range(max(0, be - retention), be)
        cur = range(bs, be)
        dsegs, specs = [], []
        for p in range(P):
            for qf in cur:
                d = []
                for kf in ret:
                    app(d, ab(p, kf), L, _temporal(qf, kf, n, window))
                if direct:
                    for o in range(P):
                        if o == p:
                            continue
                        same = labels[qf][o] == labels[qf][p]
                        for kf in cur:
                            app(d, ab(o, kf), L, same and (kf // n == qf // n))
                qg = labels[qf][p]
                for g in range(N):
                    for kf in ret:
                        app(d, lb(g, kf), KL,
                            g == qg and active[kf][g] and _temporal(qf, kf, n, window))
                dsegs.append(d)
                specs.append((ab(p, qf), L))
        for qf in cur:
            for g in range(N):
                d = []
                qa = active[qf][g]
                for p in range(P):
                    pa = qa and labels[qf][p] == g
                    for kf in ret:
                        app(d, ab(p, kf), L, pa and _temporal(qf, kf, n, window))
                for kf in ret:
                    app(d, lb(g, kf), KL, qa and active[kf][g] and _temporal(qf, kf, n, window))
                for kf in ret:
                    app(d, gb(kf), KG, qa and _temporal(qf, kf, n, window))
                dsegs.append(d)
                specs.append((lb(g, qf), KL))
        for qf in cur:
            d = []
            for g in range(N):
                for kf in ret:
                    app(d, lb(g, kf), KL, active[kf][g] and _temporal(qf, kf, n, window))
            for kf in ret:
                app(d, gb(kf), KG, _temporal(qf, kf, n, window))
            dsegs.append(d)
            specs.append((gb(qf), KG))
        out.append(pack_layout(dsegs, specs))
    return out


def tiled_cached_layout(*, P, N, L, KL, KG, n_frames, n_block, local_attn, agent, local, glob,
                        local_active, labels, q_active, direct):
    """``build_hier_tiled_cached_layout`` (``hier_tiled_attention.py:474-655``)."""
    fa, fl = len(agent[0]), len(local[0])
    lp = P * fa * L
    gp = lp + N * fl * KL
    qfs = tuple(glob[-n_frames:]) if KG > 0 else tuple(agent[0][-n_frames:])
    ab = lambda p, fi: (p * fa + fi) * L  # noqa: E731
    lb = lambda g, fi: lp + (g * fl + fi) * KL  # noqa: E731
    gb = lambda fi: gp + fi * KG  # noqa: E731

    def app(d, base, width, ok):
        d.extend((base + t, bool(ok)) for t in range(width))

    cur_idx = [tuple({f: i for i, f in enumerate(agent[p])}[f] for f in qfs) for p in range(P)]
    dsegs, specs = [], []
    for p in range(P):
        for qrel, qf in enumerate(qfs):
            d = []
            for fi, kf in enumerate(agent[p]):
                app(d, ab(p, fi), L, _temporal(qf, kf, n_block, local_attn))
            if direct:
                for o in range(P):
                    if o == p:
                        continue
                    same = labels[qrel][o] == labels[qrel][p]
                    for kr, kf in enumerate(qfs):
                        app(d, ab(o, cur_idx[o][kr]), L, same and (kf // n_block == qf // n_block))
            qg = labels[qrel][p]
            for g in range(N):
                for fi, kf in enumerate(local[g]):
                    app(d, lb(g, fi), KL,
                        g == qg and local_active[g][fi] and _temporal(qf, kf, n_block, local_attn))
            dsegs.append(d)
            specs.append((p * n_frames * L + qrel * L, L))
    aq = P * n_frames * L
    lq = n_frames * N * KL
    for qrel, qf in enumerate(qfs):
        for g in range(N):
            d = []
            qa = q_active[qrel][g]
            for p in range(P):
                pa = qa and labels[qrel][p] == g
                for fi, kf in enumerate(agent[p]):
                    app(d, ab(p, fi), L, pa and _temporal(qf, kf, n_block, local_attn))
            for fi, kf in enumerate(local[g]):
                app(d, lb(g, fi), KL,
                    qa and local_active[g][fi] and _temporal(qf, kf, n_block, local_attn))
            for fi, kf in enumerate(glob):
                app(d, gb(fi), KG, qa and _temporal(qf, kf, n_block, local_attn))
            dsegs.append(d)
            specs.append((aq + qrel * N * KL + g * KL, KL))
    for qrel, qf in enumerate(qfs):
        d = []
        for g in range(N):
            for fi, kf in enumerate(local[g]):
                app(d, lb(g, fi), KL, local_active[g][fi] and _temporal(qf, kf, n_block, local_attn))
        for fi, kf in enumerate(glob):
            app(d, gb(fi), KG, _temporal(qf, kf, n_block, local_attn))
        dsegs.append(d)
        specs.append((aq + lq + qrel * KG, KG))
    return pack_layout(dsegs, specs)


# ---------------------------------------------------------------------------
# numerics: camera Q/K add, RMSNorm, RoPE, masked softmax attention
# ---------------------------------------------------------------------------


def prologue(qx, kx, cam, wcq, wck, nqw, nkw, freqs, H, eps=1e-6):
    """fp32 restatement of ``SelfAttention._project_self_attn_qkv`` after the
    q/k projections: camera add (``attention.py:307-320``), RMSNorm over the
    full model dim (``attention.py:231-242``), then RoPE as a complex multiply
    in float64 (``rope.py:248-254``).  ``freqs`` is ``[S, D/2, 2]`` (real,
    imag) float64.  Returns fp32 ``(q, k)`` of shape ``[S, H*D]``."""
    def one(x, w_cam, w_norm):
        x = x.astype(np.float32)
        if cam is not None:
            x = x + cam.astype(np.float32) @ w_cam.astype(np.float32).T
        ms = (x.astype(np.float32) ** 2).mean(-1, keepdims=True)
        x = x / np.sqrt(ms + np.float32(eps))
        x = x * w_norm.astype(np.float32)
        S, dim = x.shape
        xc = x.astype(np.float64).reshape(S, H, dim // H // 2, 2)
        re, im = xc[..., 0], xc[..., 1]
        fr = freqs[:, None, :, 0]
        fi = freqs[:, None, :, 1]
        o = np.stack([re * fr - im * fi, re * fi + im * fr], -1)
        return o.reshape(S, dim).astype(np.float32)

    return one(qx, wcq, nqw), one(kx, wck, nkw)


def prologue_head(x, cam, w_cam, w_norm, freqs, H, head, eps=1e-6):
    """Same math as :func:`prologue` for one tensor, returning only the
    columns of ``head`` (the RMSNorm statistic still covers the full row)."""
    x = x.astype(np.float32)
    if cam is not None:
        x = x + cam.astype(np.float32) @ w_cam.astype(np.float32).T
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + np.float32(eps))
    S, dim = x.shape
    D = dim // H
    sl = slice(head * D, (head + 1) * D)
    y = (x[:, sl] * r * w_norm[sl].astype(np.float32)).astype(np.float64).reshape(S, D // 2, 2)
    fr, fi = freqs[..., 0], freqs[..., 1]
    o = np.stack([y[..., 0] * fr - y[..., 1] * fi, y[..., 0] * fi + y[..., 1] * fr], -1)
    return o.reshape(S, D).astype(np.float32)


def masked_attention(q, k, v, H, mask_rows_fn, row_chunk=1024, heads=None):
    """fp32 ``softmax(q k^T / sqrt(D) + mask) v`` per head, as SDPA with a bool
    mask (``attention.py:47-54``).  ``mask_rows_fn(r0, r1)`` returns the bool
    mask rows ``[r1-r0, S]``.  Rows whose mask is empty produce NaN in SDPA; the
    hierarchical masks never have such rows (inactive local hubs keep a self
    edge), and this oracle returns 0 there."""
    S, dim = q.shape
    D = dim // H
    hs = range(H) if heads is None else heads
    out = np.zeros((S, dim), np.float32)
    scale = np.float32(1.0 / math.sqrt(D))
    for r0 in range(0, S, row_chunk):
        r1 = min(S, r0 + row_chunk)
        m = mask_rows_fn(r0, r1)
        for h in hs:
            sl = slice(h * D, (h + 1) * D)
            s = (q[r0:r1, sl].astype(np.float32) @ k[:, sl].astype(np.float32).T) * scale
            s = np.where(m, s, -np.inf)
            mx = s.max(-1, keepdims=True)
            mx = np.where(np.isfinite(mx), mx, 0)
            p = np.exp(s - mx)
            l = p.sum(-1, keepdims=True)
            o = (p @ v[:, sl].astype(np.float32)) / np.where(l > 0, l, 1)
            out[r0:r1, sl] = np.where(l > 0, o, 0)
    return out


def segment_attention(q, k, v, H, segments):
    """fp32 attention over explicit per-segment key lists (the cached backends'
    contract, ``hier_segmented_attention.py:27-114``): rows of a segment with
    no keys produce 0."""
    S, dim = q.shape
    D = dim // H
    out = np.zeros((S, dim), np.float32)
    scale = np.float32(1.0 / math.sqrt(D))
    for q0, ql, sel in segments:
        if not sel:
            continue
        idx = np.asarray(sel)
        for h in range(H):
            sl = slice(h * D, (h + 1) * D)
            s = (q[q0:q0 + ql, sl] @ k[idx, sl].T) * scale
            s = s - s.max(-1, keepdims=True)
            p = np.exp(s)
            out[q0:q0 + ql, sl] = (p @ v[idx, sl]) / p.sum(-1, keepdims=True)
    return out


# ---------------------------------------------------------------------------
# RoPE frequency tables (rope.py:103-237) and camera12 (data/dataset.py:49-90)
# ---------------------------------------------------------------------------


def precompute_freqs(dim, end, theta=10000.0):
    """``precompute_freqs_cis`` (``rope.py:103-107``) as (cos, sin) float64."""
    f = 1.0 / theta ** (np.arange(0, dim, 2)[: dim // 2].astype(np.float64) / dim)
    ang = np.outer(np.arange(end), f)
    return np.stack([np.cos(ang), np.sin(ang)], -1)


def simplex_vertices(pool, d_agent):
    """``build_simplex_vertices`` (``rope.py:110-126``)."""
    half = d_agent // 2
    e = np.eye(pool)
    c = e - 1.0 / pool
    s = c / np.maximum(np.linalg.norm(c, axis=1, keepdims=True), 1e-12)
    out = np.zeros((pool, half), np.float32)
    out[:, :pool] = s.astype(np.float32)
    return out


def self_attn_freqs_with_hub(P, T, h, w, n_hub, head_dim, splits, pool, gamma=1.0,
                             start_frame=0, end=1024):
    """Player simplex-4D freqs (``rope.py:129-220``) followed by hub freqs
    (``rope.py:223-237``), concatenated as ``WanModel.build_self_attn_freqs_with_hub``
    does (``wan_video_dit.py:338-359``).  Returns ``[S, D/2, 2]`` float64."""
    d_t, d_a, d_h, d_w = splits
    d_t_old = head_dim - 2 * (head_dim // 3)
    ft = precompute_freqs(d_t_old, end)[:, -(d_t // 2):]
    fh = precompute_freqs(d_h, end)
    fw = precompute_freqs(d_w, end)
    verts = simplex_vertices(pool, d_a)
    parts = []
    for p in range(P):
        ang = verts[p].astype(np.float64) * gamma
        a = np.stack([np.cos(ang), np.sin(ang)], -1)
        tt = np.broadcast_to(ft[start_frame:start_frame + T][:, None, None], (T, h, w) + ft.shape[1:])
        hh = np.broadcast_to(fh[:h][None, :, None], (T, h, w) + fh.shape[1:])
        ww = np.broadcast_to(fw[:w][None, None, :], (T, h, w) + fw.shape[1:])
        aa = np.broadcast_to(a[None, None, None], (T, h, w) + a.shape)
        parts.append(np.concatenate([tt, aa, hh, ww], axis=3).reshape(T * h * w, -1, 2))
    tt = np.repeat(ft[start_frame:start_frame + T], n_hub, axis=0)
    ident = np.zeros((T * n_hub, (d_a + d_h + d_w) // 2, 2))
    ident[..., 0] = 1.0
    parts.append(np.concatenate([tt, ident], axis=1))
    return np.concatenate(parts, 0)

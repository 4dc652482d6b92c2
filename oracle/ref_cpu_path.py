"""The reference's CPU attention path, issued as the same torch calls.

TEST INFRASTRUCTURE AND TIMED CPU BASELINE ONLY.  Only ``tests/`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` import this
module; the product path (``multics_b200``) never does.

TencentARC/Multics is pure Python on torch.  Its full-sequence hierarchical
self-attention with ``attn_impl="sdpa"`` is, per layer after the q/k/v
projections (``multics/models/attention.py:355-365``):

1. camera add ``qx + cam_q(cam)``, ``kx + cam_k(cam)``
   (``attention.py:307-320``; ``CompatibleLinear`` pads the 12 camera inputs
   to 16 with zero columns, ``compatible_linear.py:12-50``, which leaves the
   product unchanged);
2. ``RMSNorm`` in fp32 over the whole model dim, times the weight
   (``attention.py:231-242``);
3. ``rope_apply``: complex multiply in float64, cast back
   (``rope.py:248-254``);
4. ``flash_attention(q, k, v, num_heads, mask=dense_bool_mask)`` =
   ``F.scaled_dot_product_attention(q, k, v, attn_mask=mask)`` per
   ``[b, n, s, d]`` head layout (``attention.py:39-54``), with the dense mask of
   ``build_stage2_hier_self_attn_mask`` (``hier_masks.py:364-641``).

The reference's package metadata does not build (setuptools stops at the
flat-layout discovery of ``asset``, ``multics`` and ``configs``), so it
cannot be installed and carried to the GPU machine.  This module issues the
same torch calls in the same order and precision (fp32, the precision the
reference's CPU oracle runs in; float64 RoPE).  Its outputs are pinned to the
reference's own outputs in ``tests/test_oracle_golden.py``.

The dense mask comes from :func:`oracle.hier_oracle.dense_mask` evaluated at
unit scale (one token per player frame, local hub and global hub) and
expanded to tokens (:func:`dense_mask_rows_units`), which is equal to the
token-level mask and fast enough to build row chunks of the full-size
configurations.
"""

from __future__ import annotations

import math
import os
import time
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from . import hier_oracle as O


def camera_add(x, cam, w_cam):
    """``x + cam @ w_cam^T`` (``attention.py:319-320``)."""
    if cam is None:
        return x
    return x + F.linear(cam.to(x.dtype), w_cam.to(x.dtype))


def rms_norm(x, weight, eps=1e-6):
    """``RMSNorm.forward`` (``attention.py:231-242``): fp32 statistic, cast
    back, then times the weight."""
    dtype = x.dtype
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).to(dtype) * weight


def rope_apply(x, freqs, num_heads):
    """``rope_apply`` (``rope.py:248-254``): ``x`` ``[b, s, n*d]``, ``freqs``
    complex ``[s, 1, d/2]``."""
    b, s, nd = x.shape
    xr = x.reshape(b, s, num_heads, nd // num_heads)
    xc = torch.view_as_complex(xr.to(torch.float64).reshape(b, s, num_heads, -1, 2))
    return torch.view_as_real(xc * freqs).flatten(3).reshape(b, s, nd).to(x.dtype)


def prologue(qx, kx, cam, wcq, wck, nqw, nkw, freqs, num_heads, eps=1e-6):
    """Steps 1-3 on ``[b, s, n*d]`` fp32 tensors; returns roped ``(q, k)``."""
    q = rope_apply(rms_norm(camera_add(qx, cam, wcq), nqw, eps), freqs, num_heads)
    k = rope_apply(rms_norm(camera_add(kx, cam, wck), nkw, eps), freqs, num_heads)
    return q, k


def sdpa_rows(q, k, v, mask_rows, num_heads, heads=None, r0=0, r1=None):
    """Step 4 for query rows ``[r0, r1)`` (all rows by default) and the given
    heads: ``q/k/v`` ``[b, s, n*d]``, ``mask_rows`` bool ``[r1-r0, s]``.
    Returns ``[b, r1-r0, len(heads)*d]``."""
    b, s, nd = q.shape
    d = nd // num_heads
    r1 = s if r1 is None else r1
    # "b s (n d) -> b n s d" as views, the layout the reference hands to SDPA
    qh, kh, vh = (t.view(b, s, num_heads, d).transpose(1, 2) for t in (q, k, v))
    if heads is None:
        sel = slice(None)
    else:
        hs = list(heads)
        sel = (slice(hs[0], hs[0] + len(hs)) if hs == list(range(hs[0], hs[0] + len(hs)))
               else torch.tensor(hs))
    qh, kh, vh = qh[:, sel, r0:r1], kh[:, sel], vh[:, sel]
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask_rows.to(torch.bool))
    return o.transpose(1, 2).reshape(b, r1 - r0, -1)


# ---------------------------------------------------------------------------
# dense mask rows by unit expansion
# ---------------------------------------------------------------------------


class UnitMask:
    """The hierarchical mask at unit scale and each token's unit, so that any
    row range of the token-level mask is ``unit[row_unit[r]][:, col_unit]``.
    The mask is uniform inside a unit pair except for an inactive local hub's
    self edge (``hier_masks.py:476-480``): a diagonal of its ``K_L`` tokens,
    restored after the expansion."""

    def __init__(self, P, T, L, N, KL, KG, n_block, local_attn, **kw):
        self.S = P * T * L + T * (N * KL + KG)
        self.unit = O.dense_mask(P, T, 1, N, 1 if KL else 0, 1 if KG else 0, n_block,
                                 local_attn, **kw)
        A = P * T * L
        tok = np.arange(self.S)
        u = np.empty(self.S, np.int64)
        u[:A] = tok[:A] // L
        if KL:
            u[A:A + T * N * KL] = P * T + (tok[A:A + T * N * KL] - A) // KL
        if KG:
            u[A + T * N * KL:] = P * T + (T * N if KL else 0) + (tok[A + T * N * KL:] - A - T * N * KL) // KG
        self.tok_unit = u
        _, active, _, _ = O.prepare_grouping(P, T, N, kw.get("labels"), kw.get("active"),
                                             kw.get("membership"), kw.get("global_only"))
        # tokens of inactive local hubs: their own unit block is the diagonal
        self.inactive_local = np.zeros(self.S, bool)
        if KL:
            for t in range(T):
                for g in range(N):
                    if not active[t, g]:
                        a = A + (t * N + g) * KL
                        self.inactive_local[a:a + KL] = True

    def rows(self, r0, r1):
        m = self.unit[self.tok_unit[r0:r1]][:, self.tok_unit]
        ri = np.nonzero(self.inactive_local[r0:r1])[0]
        if ri.size:
            own = self.tok_unit[r0 + ri]
            for i, u in zip(ri, own):
                cols = np.nonzero(self.tok_unit == u)[0]
                m[i, cols] = False
                m[i, r0 + i] = bool(self.unit[u, u])
        return m


def dense_mask_rows_units(P, T, L, N, KL, KG, n_block, local_attn, rows: slice, **kw):
    """Rows ``rows`` of the dense mask by unit expansion (equal to
    :func:`oracle.hier_oracle.dense_mask` with ``rows``)."""
    um = UnitMask(P, T, L, N, KL, KG, n_block, local_attn, **kw)
    r0, r1, _ = rows.indices(um.S)
    return um.rows(r0, r1)


# ---------------------------------------------------------------------------
# timed CPU baseline over a full-size configuration
# ---------------------------------------------------------------------------


class RefCPULayer:
    """One hierarchical attention layer of a configuration, run through the
    reference's CPU path on the host cores in fp32.

    The prologue (steps 1-3) runs once over the whole layer and is timed.
    Attention (step 4) is timed in work units of one head over a 512-row
    chunk of queries against all keys: the units are visited chunk-strided
    (consecutive units lie far apart in the sequence, so a prefix of the
    visit order samples the whole layer) and head by head.  The reported rate
    is useful FLOPs (4*D per unmasked pair per head) over the attention time
    of the sampled units plus their share of the prologue time.  The dense
    mask is built per grouping, outside the timed region, as the GPU path
    builds its plans outside its timed region."""

    def __init__(self, cfg, threads: Optional[int] = None, chunk: int = 512):
        from multics_b200.synth import make_inputs

        self.threads = threads or os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.cfg = cfg
        self.chunk = chunk
        inp = make_inputs(cfg, device="cpu")
        labels = inp.labels.numpy()
        self.mask = UnitMask(cfg.P, cfg.T, cfg.L, cfg.N, cfg.KL, cfg.KG, cfg.n_block,
                             cfg.local_attn, labels=labels, direct=cfg.direct)
        f32 = lambda t: t.float().unsqueeze(0)  # noqa: E731
        t0 = time.perf_counter()
        with torch.no_grad():
            self.q, self.k = prologue(f32(inp.qx), f32(inp.kx), f32(inp.cam), inp.wcq.float(),
                                      inp.wck.float(), inp.nqw.float(), inp.nkw.float(),
                                      inp.freqs, cfg.H)
        self.prologue_s = time.perf_counter() - t0
        self.v = f32(inp.v)
        self.S = cfg.S
        self.n_chunks = -(-self.S // chunk)
        stride = 37
        while math.gcd(stride, self.n_chunks) != 1:
            stride += 2
        self.visit = [(i * stride) % self.n_chunks for i in range(self.n_chunks)]
        self.cursor = 0
        self._mask_cache = {}

    def _mask_rows(self, c):
        m = self._mask_cache.get(c)
        if m is None:
            r0 = c * self.chunk
            m = torch.from_numpy(self.mask.rows(r0, min(self.S, r0 + self.chunk)))
            if len(self._mask_cache) > 96:
                self._mask_cache.pop(next(iter(self._mask_cache)))
            self._mask_cache[c] = m
        return m

    def sample(self, seconds: float):
        """Run work units for about ``seconds`` of attention time; returns
        ``(useful_flops, seconds_including_prologue_share, units, rows)``."""
        cfg = self.cfg
        flops, el, units, rows = 0.0, 0.0, 0, 0
        while el < seconds:
            i = self.cursor % (self.n_chunks * cfg.H)
            head, c = i // self.n_chunks, self.visit[i % self.n_chunks]
            m = self._mask_rows(c)
            r0 = c * self.chunk
            r1 = r0 + m.shape[0]
            t = time.perf_counter()
            with torch.no_grad():
                sdpa_rows(self.q, self.k, self.v, m, cfg.H, heads=[head], r0=r0, r1=r1)
            dt = time.perf_counter() - t
            share = self.prologue_s * (r1 - r0) / (self.S * cfg.H)
            el += dt + share
            flops += 4.0 * cfg.D * float(m.sum())
            units += 1
            rows += r1 - r0
            self.cursor += 1
        return flops, el, units, rows

    def describe(self, units, rows):
        return (f"reference CPU path as torch calls (fp32 camera add + RMSNorm, float64 RoPE, "
                f"F.scaled_dot_product_attention with the dense bool mask), {self.threads} "
                f"threads: {units} units of one head x 512 query rows ({rows} rows) of the "
                f"full {self.cfg.name} layer, chunk-strided over the sequence, plus their share "
                f"of the whole-layer prologue ({self.prologue_s:.2f} s); useful FLOP/s = "
                f"4*D*unmasked pairs / time")


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# action branch of the DiT block (test infrastructure only)
# ---------------------------------------------------------------------------


def temporal_block_causal_mask(num_frames, num_frame_per_block, local_attn_size):
    """``get_temporal_block_causal_mask`` (``hier_masks.py:1152-1166``), in
    numpy: frame ``i`` sees frame ``j`` iff ``j // n <= i // n`` and, with a
    window, ``i - j < local_attn_size``."""
    t = np.arange(num_frames)
    m = (t[None, :] // num_frame_per_block) <= (t[:, None] // num_frame_per_block)
    if local_attn_size != -1:
        m &= (t[:, None] - t[None, :]) < local_attn_size
    return m


def keyboard_mask(frame_mask, num_patches, tokens_per_kbd_frame=12):
    """``repeat(frame_mask, "f g -> (f q) (g k)")`` (``blocks.py:446-448``)."""
    return np.repeat(np.repeat(np.asarray(frame_mask), num_patches, 0), tokens_per_kbd_frame, 1)


def shared_mask_sdpa(q, k, v, num_heads, mask):
    """``flash_attention(q, k, v, num_heads, mask)`` (``attention.py:47-54``)
    with one mask ``[Lq, Lk]`` broadcast over the batch: ``q`` ``[B, Lq,
    n*d]``, ``k``/``v`` ``[B, Lk, n*d]``."""
    B, Lq, nd = q.shape
    d = nd // num_heads
    qh, kh, vh = (t.reshape(B, t.shape[1], num_heads, d).transpose(1, 2) for t in (q, k, v))
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=torch.as_tensor(mask).to(torch.bool))
    return o.transpose(1, 2).reshape(B, Lq, nd)


def action_temporal_forward(x, w, num_heads, mask, eps=1e-6):
    """The per-frame action attention, a ``SelfAttention`` over ``x``
    ``[B, F, dim]`` (``blocks.py:677-691``, ``attention.py:355-365,436-442``):
    q/k/v linears, RMSNorm on q and k, 1-D RoPE over the frames
    (``precompute_freqs_cis(head_dim, F)``), masked SDPA, output linear.
    ``w`` maps ``q.weight``, ``q.bias``, ... ``norm_k.weight`` to tensors."""
    B, F_, dim = x.shape
    d = dim // num_heads
    q = rms_norm(F.linear(x, w["q.weight"], w["q.bias"]), w["norm_q.weight"], eps)
    k = rms_norm(F.linear(x, w["k.weight"], w["k.bias"]), w["norm_k.weight"], eps)
    v = F.linear(x, w["v.weight"], w["v.bias"])
    cs = torch.from_numpy(O.precompute_freqs(d, F_))
    freqs = torch.complex(cs[..., 0], cs[..., 1]).unsqueeze(1)
    q, k = rope_apply(q, freqs, num_heads), rope_apply(k, freqs, num_heads)
    o = shared_mask_sdpa(q, k, v, num_heads, mask)
    return F.linear(o, w["o.weight"], w["o.bias"])


def action_cross_forward(x, ctx, w, num_heads, mask, eps=1e-6):
    """The keyboard cross-attention, a ``CrossAttention`` without image input
    (``attention.py:1071-1090``): q from ``x``, k/v from ``ctx``, RMSNorm on
    q and k, masked SDPA, output linear."""
    q = rms_norm(F.linear(x, w["q.weight"], w["q.bias"]), w["norm_q.weight"], eps)
    k = rms_norm(F.linear(ctx, w["k.weight"], w["k.bias"]), w["norm_k.weight"], eps)
    v = F.linear(ctx, w["v.weight"], w["v.bias"])
    o = shared_mask_sdpa(q, k, v, num_heads, mask)
    return F.linear(o, w["o.weight"], w["o.bias"])

"""RoPE frequency tables for the hierarchical sequence (host side, torch).

Same functions and outputs as the reference's ``multics/models/rope.py``
(complex128 multipliers): Wan 1-D tables, regular-simplex agent vertices,
the 4-D (t, agent, h, w) per-player tables and the hub tables, concatenated
in the order ``WanModel.build_self_attn_freqs_with_hub`` uses
(``multics/models/wan_video_dit.py:338-359``).
"""

from __future__ import annotations

from typing import Sequence, Tuple

import torch

WAN_REROPE_SPLITS = (12, 32, 42, 42)


def precompute_freqs_cis(dim: int, end: int = 1024, theta: float = 10000.0):
    """``rope.py:103-107``."""
    freqs = 1.0 / theta ** (torch.arange(0, dim, 2)[: dim // 2].double() / dim)
    freqs = torch.outer(torch.arange(end, device=freqs.device), freqs)
    return torch.polar(torch.ones_like(freqs), freqs)


def build_simplex_vertices(pool_size: int, d_agent: int) -> torch.Tensor:
    """Regular simplex vertices ``[pool, d_agent//2]`` (``rope.py:110-126``)."""
    m = int(pool_size)
    half = d_agent // 2
    if m < 2:
        raise ValueError("pool_size must be >= 2")
    if m > half + 1:
        raise ValueError(f"pool_size {m} exceeds limit d_agent//2+1={half + 1} for d_agent={d_agent}")
    e = torch.eye(m, dtype=torch.float64)
    centered = e - 1.0 / m
    s = centered / centered.norm(dim=1, keepdim=True).clamp(min=1e-12)
    out = torch.zeros(m, half, dtype=torch.float32)
    out[:, :m] = s.to(torch.float32)
    return out


def precompute_freqs_cis_4d_wan_rerope(head_dim: int = 128, end: int = 1024,
                                       theta: float = 10000.0,
                                       splits: Tuple[int, int, int, int] = WAN_REROPE_SPLITS):
    """``rope.py:129-144``."""
    d_t, d_a, d_h, d_w = splits
    assert d_t + d_a + d_h + d_w == head_dim, splits
    d_t_old = head_dim - 2 * (head_dim // 3)
    freqs_t = precompute_freqs_cis(d_t_old, end, theta)[:, -(d_t // 2):]
    return {"t": freqs_t, "h": precompute_freqs_cis(d_h, end, theta),
            "w": precompute_freqs_cis(d_w, end, theta), "splits": splits, "d_a": d_a}


def build_multiplayer_freqs_4d(bands, f, h, w, agent_vertex_ids: Sequence[int],
                               simplex_vertices, gamma=1.0, device=None, start_frame=0):
    """Player-major ``[P*f*h*w, 1, D/2]`` tables (``rope.py:155-220``)."""
    d_t, d_a, d_h, d_w = bands["splits"]
    n_t, n_h, n_w = d_t // 2, d_h // 2, d_w // 2
    ft = bands["t"][start_frame:start_frame + f].to(device)
    fh = bands["h"][:h].to(device)
    fw = bands["w"][:w].to(device)
    thw = torch.cat([ft.view(f, 1, 1, n_t).expand(f, h, w, n_t),
                     fh.view(1, h, 1, n_h).expand(f, h, w, n_h),
                     fw.view(1, 1, w, n_w).expand(f, h, w, n_w)], -1).reshape(f * h * w, -1)
    parts = []
    for vid in agent_vertex_ids:
        ang = simplex_vertices[int(vid)].to(torch.float64) * float(gamma)
        a = torch.polar(torch.ones_like(ang), ang).to(device).view(1, -1).expand(f * h * w, -1)
        parts.append(torch.cat([thw[:, :n_t], a, thw[:, n_t:]], -1).unsqueeze(1))
    return torch.cat(parts, 0)


def build_hub_freqs_4d(bands, f, num_hub_tokens, start_frame=0, device=None):
    """Hub tables: temporal phase only (``rope.py:223-237``)."""
    d_t, d_a, d_h, d_w = bands["splits"]
    ft = bands["t"][start_frame:start_frame + f].to(device)
    t_grid = ft.repeat_interleave(num_hub_tokens, dim=0)
    ident = torch.ones(f * num_hub_tokens, (d_a + d_h + d_w) // 2, device=device,
                       dtype=torch.complex64)
    return torch.cat([t_grid, ident], -1).unsqueeze(1)


def self_attn_freqs_with_hub(P, f, h, w, num_hub_tokens, head_dim=128, splits=WAN_REROPE_SPLITS,
                             pool_size=10, gamma=1.0, agent_vertex_ids=None, start_frame=0,
                             device=None):
    """Full-sequence table ``[P*f*h*w + f*num_hub_tokens, 1, D/2]`` complex128."""
    bands = precompute_freqs_cis_4d_wan_rerope(head_dim, splits=splits)
    verts = build_simplex_vertices(pool_size, splits[1])
    ids = list(range(P)) if agent_vertex_ids is None else list(agent_vertex_ids)
    a = build_multiplayer_freqs_4d(bands, f, h, w, ids, verts, gamma, device, start_frame)
    hub = build_hub_freqs_4d(bands, f, num_hub_tokens, start_frame, device)
    return torch.cat([a, hub], 0)

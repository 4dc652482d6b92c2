"""Seeded synthetic inputs with the benchmark configurations' shapes.

The reference measures on real multi-player clips; these stand-ins have the
same shapes and value distributions: projected q/k/v ~ N(0,1)*scale, per
player/frame random SE(3) camera poses converted to the model's camera12
representation, N(0,0.02) camera adapter weights, 1+N(0,0.02) RMSNorm
weights, simplex-4D RoPE tables.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

from .rope import self_attn_freqs_with_hub


@dataclass
class HierConfig:
    name: str
    P: int
    T: int
    h: int
    w: int
    N: int
    KL: int
    KG: int
    H: int = 24
    D: int = 128
    n_block: int = 1
    local_attn: int = -1
    direct: bool = True
    groups: Optional[list] = None       # static labels row (player -> group)
    regroup_every: int = 0              # >0: seeded permutation per segment
    page_size: int = 0                  # >0: paged K/V pool with shuffled pages
    scale: float = 0.5
    seed: int = 0

    @property
    def L(self):
        return self.h * self.w

    @property
    def S(self):
        return self.P * self.T * self.L + self.T * (self.N * self.KL + self.KG)

    @property
    def dim(self):
        return self.H * self.D


CONFIGS = {
    # config 2: one full-size layer, 4 players x 42 frames x 220 tokens
    "cfg2": HierConfig("cfg2", P=4, T=42, h=11, w=20, N=2, KL=16, KG=6, groups=[0, 0, 1, 1]),
    # config 4: 8 players, 4 groups of 2 re-permuted every 3 latent frames
    "cfg4": HierConfig("cfg4", P=8, T=42, h=11, w=20, N=4, KL=16, KG=6, regroup_every=3),
    # config 5: 10 players in groups (3,3,2,2), 64-token pages shuffled by seed
    "cfg5": HierConfig("cfg5", P=10, T=42, h=11, w=20, N=4, KL=16, KG=6,
                       groups=[0, 0, 0, 1, 1, 1, 2, 2, 3, 3], page_size=64),
    # config 1 shape with head_dim 128 (CPU-checkable)
    "cfg1": HierConfig("cfg1", P=4, T=3, h=4, w=4, N=2, KL=8, KG=6, H=2, groups=[0, 0, 1, 1],
                       scale=1.0),
}


def group_labels(cfg: HierConfig, generator: torch.Generator) -> torch.Tensor:
    """``[T,P]`` int64 labels for the config."""
    if cfg.regroup_every > 0:
        rows = []
        per = cfg.P // cfg.N
        for t0 in range(0, cfg.T, cfg.regroup_every):
            perm = torch.randperm(cfg.P, generator=generator)
            row = torch.empty(cfg.P, dtype=torch.long)
            row[perm] = torch.arange(cfg.P) // per
            rows += [row] * min(cfg.regroup_every, cfg.T - t0)
        return torch.stack(rows)
    return torch.tensor([cfg.groups] * cfg.T, dtype=torch.long)


def euler_zyx(ang: torch.Tensor) -> torch.Tensor:
    z, y, x = ang[..., 0], ang[..., 1], ang[..., 2]
    cz, sz, cy, sy, cx, sx = z.cos(), z.sin(), y.cos(), y.sin(), x.cos(), x.sin()
    R = torch.stack([
        torch.stack([cz * cy, cz * sy * sx - sz * cx, cz * sy * cx + sz * sx], -1),
        torch.stack([sz * cy, sz * sy * sx + cz * cx, sz * sy * cx - cz * sx], -1),
        torch.stack([-sy, cy * sx, cy * cx], -1)], -2)
    return R


def camera12_from_c2w(c2w: torch.Tensor, pos_scale: float = 1.0) -> torch.Tensor:
    """Absolute ``[P,T,4,4]`` camera-to-world -> ``[P,T,12]`` relative to player 0
    frame 0 (the representation of ``multics/data/dataset.py:49-90``)."""
    c2w = c2w.to(torch.float64)
    anchor = c2w[0, 0]
    w2c = torch.eye(4, dtype=torch.float64)
    w2c[:3, :3] = anchor[:3, :3].T
    w2c[:3, 3] = -(anchor[:3, :3].T @ anchor[:3, 3])
    rel = w2c.view(1, 1, 4, 4) @ c2w
    rel[..., :3, 3] /= float(pos_scale)
    return rel[..., :3, :].reshape(c2w.shape[0], c2w.shape[1], 12).float()


def camera_tokens(cfg: HierConfig, generator: torch.Generator) -> torch.Tensor:
    """Per-token camera12 ``[S,12]``: player tokens broadcast over patches, hub rows 0."""
    ang = (torch.rand(cfg.P, cfg.T, 3, generator=generator, dtype=torch.float64) * 2 - 1) * math.pi
    trans = torch.randn(cfg.P, cfg.T, 3, generator=generator, dtype=torch.float64)
    c2w = torch.zeros(cfg.P, cfg.T, 4, 4, dtype=torch.float64)
    c2w[..., :3, :3] = euler_zyx(ang)
    c2w[..., :3, 3] = trans
    c2w[..., 3, 3] = 1.0
    cam12 = camera12_from_c2w(c2w)
    cam = torch.zeros(cfg.S, 12)
    cam[: cfg.P * cfg.T * cfg.L] = cam12.repeat_interleave(cfg.L, dim=1).reshape(-1, 12)
    return cam


@dataclass
class LayerInputs:
    qx: torch.Tensor
    kx: torch.Tensor
    v: torch.Tensor
    cam: torch.Tensor
    wcq: torch.Tensor
    wck: torch.Tensor
    nqw: torch.Tensor
    nkw: torch.Tensor
    freqs: torch.Tensor   # complex128 [S,1,D/2]
    labels: torch.Tensor  # [T,P]
    extra: dict = field(default_factory=dict)


def make_inputs(cfg: HierConfig, device="cpu") -> LayerInputs:
    """Seeded inputs of one hierarchical attention layer (bf16 except freqs)."""
    g = torch.Generator().manual_seed(cfg.seed)
    bf = torch.bfloat16

    def normal(*shape, scale=1.0):
        # generate in chunks to bound host memory for full-size configs
        out = torch.empty(*shape, dtype=bf)
        flat = out.view(-1)
        step = 1 << 24
        for i in range(0, flat.numel(), step):
            n = min(step, flat.numel() - i)
            flat[i:i + n] = (torch.randn(n, generator=g) * scale).to(bf)
        return out.to(device)

    qx = normal(cfg.S, cfg.dim, scale=cfg.scale)
    kx = normal(cfg.S, cfg.dim, scale=cfg.scale)
    v = normal(cfg.S, cfg.dim, scale=cfg.scale)
    cam = camera_tokens(cfg, g).to(bf).to(device)
    wcq = (torch.randn(cfg.dim, 12, generator=g) * 0.02).to(bf).to(device)
    wck = (torch.randn(cfg.dim, 12, generator=g) * 0.02).to(bf).to(device)
    nqw = (1 + 0.02 * torch.randn(cfg.dim, generator=g)).to(bf).to(device)
    nkw = (1 + 0.02 * torch.randn(cfg.dim, generator=g)).to(bf).to(device)
    freqs = self_attn_freqs_with_hub(cfg.P, cfg.T, cfg.h, cfg.w, cfg.N * cfg.KL + cfg.KG,
                                     cfg.D, pool_size=max(10, cfg.P) if cfg.P <= 17 else cfg.P)
    labels = group_labels(cfg, g)
    return LayerInputs(qx, kx, v, cam, wcq, wck, nqw, nkw, freqs.to(device), labels.to(device))


def page_table(cfg: HierConfig) -> torch.Tensor:
    """int32 logical page -> physical page of the player rows (64-token pages
    for ``cfg.page_size``), a permutation shuffled by the config's seed."""
    size = cfg.page_size or 64
    n = -(-cfg.P * cfg.T * cfg.L // size)
    g = torch.Generator().manual_seed(cfg.seed + 1)
    return torch.randperm(n, generator=g).to(torch.int32)


def cached_step_inputs(P=4, N=2, L=220, KL=16, KG=6, n_frames=3, local_attn=21, retained=24,
                       H=24, device="cuda", seed=0) -> dict:
    """Keyword arguments of the cached-backend plugin
    (``multics_b200.cached.hierarchical_cached_attention``) for one block of
    ``n_frames`` new frames against rolling caches holding ``retained``
    frames per stream (the released inference shape: 4 players, 3-frame
    blocks, window 21 + 3 retained frames), with seeded random roped queries
    and cache contents ~ N(0,1)*0.5, groups {0,1},{2,3} and every hub active."""
    g = torch.Generator().manual_seed(seed)
    dim = H * 128
    S = P * n_frames * L + n_frames * (N * KL + KG)
    fr = torch.arange(retained, dtype=torch.int64)

    def frames(w):
        return fr.repeat_interleave(max(w, 1)).to(device)

    def rnd(rows):
        return (torch.randn((1, rows, dim), generator=g) * 0.5).to(torch.bfloat16).to(device)

    kw = dict(P=P, N=N, L=L, KL=KL, KG=KG, n_frames=n_frames, n_block=n_frames,
              local_attn=local_attn, direct_player=True, hier_no_local_hub=False)
    kw["agent_frames"] = [frames(L) for _ in range(P)]
    kw["agent_keys"] = [rnd(retained * L) for _ in range(P)]
    kw["agent_vals"] = [rnd(retained * L) for _ in range(P)]
    kw["local_frames"] = [frames(KL) for _ in range(N)]
    kw["local_keys"] = [rnd(retained * KL) for _ in range(N)]
    kw["local_vals"] = [rnd(retained * KL) for _ in range(N)]
    kw["local_active_tokens"] = [torch.ones(retained * KL, dtype=torch.bool, device=device)
                                 for _ in range(N)]
    kw["global_frames"] = frames(KG)
    kw["global_keys"] = rnd(retained * KG)
    kw["global_vals"] = rnd(retained * KG)
    kw["labels"] = torch.tensor([[p * N // P for p in range(P)]] * n_frames, dtype=torch.long,
                                device=device)
    kw["active"] = torch.ones((n_frames, N), dtype=torch.bool, device=device)
    kw["roped_q"] = (torch.randn((1, S, H, 128), generator=g) * 0.5).to(torch.bfloat16).to(device)
    return kw

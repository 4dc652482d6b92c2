"""One denoising step of a Multics-shaped DiT with the B200 hierarchical
attention in every block (benchmark configuration 3).

The reference model is Wan2.2-TI2V-5B with Multics' multi-player additions
(``multics/checkpoint.py:13-69``, ``multics/models/wan_video_dit.py:420-757``,
``multics/models/blocks.py:587-700``): per block, adaLN modulation per latent
frame, hierarchical self-attention over ``[players | hub tokens]`` with the
camera Q/K adapters, text cross-attention, an action MLP over the mouse
features, a per-frame (temporal) action attention, a keyboard cross-attention
and the FFN.  This module rebuilds that block at the same shapes around
``multics_b200.attention.SelfAttention`` (the hierarchical self-attention and,
over a batch of frame sequences, the action temporal attention) and
``multics_b200.attention.CrossAttention`` (the keyboard cross-attention), so
that the step time, and the share of each attention in it, can be measured
on B200.  Weights are random (N(0, 0.02)), as no checkpoint is available;
the GEMMs, norms and the unmasked text cross-attention run on cuBLAS and
PyTorch's SDPA, the part of the step this library does not replace.
``DiTConfig.action_impl = "sdpa"`` runs the action branch on SDPA instead, as
the reference's ``flash_attention(mask)`` does.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import CrossAttention, RMSNorm, SelfAttention, freqs_table
from .hier_masks import build_stage2_hier_flex_block_mask

__all__ = ["DiTConfig", "HierDiTBlock", "HierDiT", "dit_inputs"]


@dataclass
class DiTConfig:
    """Shape of benchmark configuration 3 (``DIT_CONFIG`` of the reference)."""

    blocks: int = 30
    dim: int = 3072
    ffn: int = 14336
    heads: int = 24
    in_dim: int = 48
    out_dim: int = 48
    text_dim: int = 4096
    text_len: int = 512
    freq_dim: int = 256
    patch: tuple = (1, 2, 2)
    players: int = 4
    frames: int = 42
    height: int = 22
    width: int = 40
    groups: tuple = (0, 0, 1, 1)
    n_groups: int = 2
    local_hub: int = 16
    global_hub: int = 6
    cam_dim: int = 12
    kb_dim: int = 23
    mouse_dim: int = 2
    kb_rows: int = 12       # keyboard / mouse rows per latent frame (3 frames x 4 sub-steps)
    eps: float = 1e-6
    action_impl: str = "b200"  # "b200" (shared-mask tcgen05 plans) or "sdpa"

    @property
    def tokens_per_frame(self) -> int:
        return (self.height // self.patch[1]) * (self.width // self.patch[2])

    @property
    def hub_per_frame(self) -> int:
        return self.n_groups * self.local_hub + self.global_hub

    @property
    def S(self) -> int:
        return self.players * self.frames * self.tokens_per_frame + self.frames * self.hub_per_frame


def _modulate(x, shift, scale):
    return x * (1 + scale) + shift


def _frame_mod(mod, L):
    """[P, F, dim] per-frame modulation -> [P, F*L, dim] per token."""
    P, Fr, d = mod.shape
    return mod[:, :, None, :].expand(P, Fr, L, d).reshape(P, Fr * L, d)


class _CrossAttention(nn.Module):
    """Query tokens attend to context tokens (text or keyboard), RMSNorm on q
    and k, optional bool mask; PyTorch SDPA."""

    def __init__(self, dim, heads, eps):
        super().__init__()
        self.heads = heads
        self.q, self.k, self.v, self.o = (nn.Linear(dim, dim) for _ in range(4))
        self.norm_q, self.norm_k = RMSNorm(dim, eps), RMSNorm(dim, eps)

    def forward(self, x, ctx, mask=None):
        B, Lq, d = x.shape
        h = self.heads
        q = self.norm_q(self.q(x)).view(B, Lq, h, d // h).transpose(1, 2)
        k = self.norm_k(self.k(ctx)).view(B, ctx.shape[1], h, d // h).transpose(1, 2)
        v = self.v(ctx).view(B, ctx.shape[1], h, d // h).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return self.o(o.transpose(1, 2).reshape(B, Lq, d))


class _FrameAttention(nn.Module):
    """Attention along the latent frames of each spatial token (the action
    temporal branch): RMSNorm q/k, 1-D RoPE over frames, block-causal frame
    mask; PyTorch SDPA over ``P*L`` short sequences."""

    def __init__(self, dim, heads, eps):
        super().__init__()
        self.heads = heads
        self.q, self.k, self.v, self.o = (nn.Linear(dim, dim) for _ in range(4))
        self.norm_q, self.norm_k = RMSNorm(dim, eps), RMSNorm(dim, eps)

    @staticmethod
    def _rope(x, cos, sin):
        x1, x2 = x[..., 0::2], x[..., 1::2]
        return torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], -1).flatten(-2)

    def forward(self, x, mask, cos, sin):
        B, Fr, d = x.shape
        h = self.heads
        q = self.norm_q(self.q(x)).view(B, Fr, h, d // h).transpose(1, 2)
        k = self.norm_k(self.k(x)).view(B, Fr, h, d // h).transpose(1, 2)
        v = self.v(x).view(B, Fr, h, d // h).transpose(1, 2)
        q, k = self._rope(q, cos, sin).to(v.dtype), self._rope(k, cos, sin).to(v.dtype)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        return self.o(o.transpose(1, 2).reshape(B, Fr, d))


class HierDiTBlock(nn.Module):
    """One block at the reference's shapes; the self-attention is this
    library's hierarchical attention (``SelfAttention.forward`` with the
    grouping's block mask)."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        d = cfg.dim
        self.cfg = cfg
        self.modulation = nn.Parameter(torch.randn(1, 1, 6, d) / d ** 0.5)
        self.norm1 = nn.LayerNorm(d, eps=cfg.eps, elementwise_affine=False)
        self.norm2 = nn.LayerNorm(d, eps=cfg.eps, elementwise_affine=False)
        self.norm3 = nn.LayerNorm(d, eps=cfg.eps)
        self.self_attn = SelfAttention(d, cfg.heads, eps=cfg.eps)
        self.self_attn.enable_camera_pose_qk(cfg.cam_dim, dropout_p=0.0)
        self.cross_attn = _CrossAttention(d, cfg.heads, cfg.eps)
        m = cfg.mouse_dim * cfg.kb_rows
        self.action_mlp = nn.Sequential(nn.LayerNorm(d + m), nn.Linear(d + m, d + m), nn.GELU(),
                                        nn.Linear(d + m, d), nn.LayerNorm(d))
        if cfg.action_impl == "b200":
            self.action_temporal_attn = SelfAttention(d, cfg.heads, eps=cfg.eps)
            self.action_cross_attn = CrossAttention(d, cfg.heads, eps=cfg.eps)
        elif cfg.action_impl == "sdpa":
            self.action_temporal_attn = _FrameAttention(d, cfg.heads, cfg.eps)
            self.action_cross_attn = _CrossAttention(d, cfg.heads, cfg.eps)
        else:
            raise ValueError(f"action_impl must be 'b200' or 'sdpa', got {cfg.action_impl!r}")
        self.ffn = nn.Sequential(nn.Linear(d, cfg.ffn), nn.GELU(approximate="tanh"),
                                 nn.Linear(cfg.ffn, d))

    def forward(self, x, x_hub, ctx, mouse, kb, t_mod, freqs, mask, cam, frame_mask, kb_mask,
                rope_f, events=None):
        """x ``[P, F*L, d]`` player tokens, x_hub ``[1, F*K, d]`` hub tokens,
        t_mod ``[P, F, 6, d]``; returns the updated ``(x, x_hub)``.
        ``events`` (six CUDA events, optional) bracket the hierarchical
        self-attention, the action temporal attention and the keyboard
        cross-attention."""
        cfg = self.cfg
        P, FL, d = x.shape
        Fr = cfg.frames
        L = FL // Fr
        K = x_hub.shape[1] // Fr
        mod = (self.modulation + t_mod).unbind(2)  # 6 x [P, F, d]
        sh_a, sc_a, g_a, sh_m, sc_m, g_m = (_frame_mod(m_, L) for m_ in mod)
        hub_mod = [_frame_mod(m_[:1], K) for m_ in mod[:3]]
        # hierarchical self-attention over [players | hubs]
        xa = _modulate(self.norm1(x), sh_a, sc_a).reshape(1, P * FL, d)
        ha = _modulate(self.norm1(x_hub), hub_mod[0], hub_mod[1])
        if events is not None:
            events[0].record()
        out = self.self_attn(torch.cat([xa, ha], 1), freqs, mask, cam)
        if events is not None:
            events[1].record()
        x = x + g_a * out[:, :P * FL].reshape(P, FL, d)
        x_hub = x_hub + hub_mod[2] * out[:, P * FL:]
        # text cross-attention
        x = x + self.cross_attn(self.norm3(x), ctx)
        # action branches: mouse MLP, per-frame attention, keyboard cross-attention
        a = self.action_mlp(torch.cat([_modulate(self.norm2(x), sh_m, sc_m), mouse], -1))
        a = a.reshape(P, Fr, L, d).transpose(1, 2).reshape(P * L, Fr, d)
        if events is not None:
            events[2].record()
        if isinstance(self.action_temporal_attn, SelfAttention):
            a = self.action_temporal_attn(a, rope_f[2], frame_mask)
        else:
            a = self.action_temporal_attn(a, frame_mask, rope_f[0], rope_f[1])
        if events is not None:
            events[3].record()
        x = x + a.reshape(P, L, Fr, d).transpose(1, 2).reshape(P, FL, d)
        xk = self.norm3(x)
        if events is not None:
            events[4].record()
        xk = self.action_cross_attn(xk, kb, kb_mask)
        if events is not None:
            events[5].record()
        x = x + xk
        # FFN
        x = x + g_m * self.ffn(_modulate(self.norm2(x), sh_m, sc_m))
        return x, x_hub


def _sinusoidal(dim, t):
    half = dim // 2
    f = torch.pow(10000.0, -torch.arange(half, dtype=torch.float64, device=t.device) / half)
    a = t.double()[:, None] * f[None]
    return torch.cat([torch.cos(a), torch.sin(a)], -1).float()


class HierDiT(nn.Module):
    """Embeddings + ``cfg.blocks`` blocks + head; ``forward`` is one
    denoising step (one model evaluation) of all players."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        d = cfg.dim
        self.cfg = cfg
        pt, ph, pw = cfg.patch
        self.patch_embedding = nn.Linear(cfg.in_dim * pt * ph * pw, d)
        self.text_embedding = nn.Sequential(nn.Linear(cfg.text_dim, d), nn.GELU(approximate="tanh"),
                                            nn.Linear(d, d))
        self.time_embedding = nn.Sequential(nn.Linear(cfg.freq_dim, d), nn.SiLU(), nn.Linear(d, d))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(d, 6 * d))
        self.keyboard_embedding = nn.Linear(cfg.kb_dim, d)
        self.hub_embedding = nn.Parameter(torch.randn(cfg.hub_per_frame, d) * 0.02)
        self.blocks = nn.ModuleList(HierDiTBlock(cfg) for _ in range(cfg.blocks))
        self.head_norm = nn.LayerNorm(d, eps=cfg.eps, elementwise_affine=False)
        self.head_modulation = nn.Parameter(torch.randn(1, 1, 2, d) / d ** 0.5)
        self.head = nn.Linear(d, cfg.out_dim * pt * ph * pw)

    def prepare(self, inputs, device):
        """Per-step constants that depend only on the grouping and shapes:
        the block mask (and the work plan built with it), RoPE tables, camera
        tokens and the action masks."""
        from .rope import self_attn_freqs_with_hub

        cfg = self.cfg
        Fr, L, K, P = cfg.frames, cfg.tokens_per_frame, cfg.hub_per_frame, cfg.players
        labels = torch.tensor([list(cfg.groups)] * Fr, device=device)
        mask, _, _ = build_stage2_hier_flex_block_mask(P, Fr, L, cfg.n_groups, cfg.local_hub,
                                                       cfg.global_hub, 1, -1, labels, None, True,
                                                       device)
        freqs = freqs_table(self_attn_freqs_with_hub(
            P, Fr, cfg.height // cfg.patch[1], cfg.width // cfg.patch[2], K, cfg.dim // cfg.heads,
            pool_size=max(10, P)).to(device))
        cam = torch.zeros(1, cfg.S, cfg.cam_dim, device=device, dtype=torch.bfloat16)
        cam[0, :P * Fr * L] = inputs["camera"].to(device, torch.bfloat16)[:, :, None, :] \
            .expand(P, Fr, L, cfg.cam_dim).reshape(-1, cfg.cam_dim)
        t = torch.arange(Fr, device=device)
        frame_mask = t[None, :] <= t[:, None]  # block-causal, one frame per block
        kb_mask = frame_mask.repeat_interleave(L, 0).repeat_interleave(cfg.kb_rows, 1)
        hd = cfg.dim // cfg.heads
        ang = t.double()[:, None] * torch.pow(10000.0, -torch.arange(0, hd, 2, device=device,
                                                                     dtype=torch.float64) / hd)
        rope_f = (ang.cos().float(), ang.sin().float(), torch.polar(torch.ones_like(ang), ang)
                  .unsqueeze(1))
        return dict(mask=mask, freqs=freqs, cam=cam, frame_mask=frame_mask, kb_mask=kb_mask,
                    rope_f=rope_f)

    def forward(self, inputs, consts, attn_events=None):
        cfg = self.cfg
        P, Fr, L = cfg.players, cfg.frames, cfg.tokens_per_frame
        d = cfg.dim
        lat = inputs["latents"]  # [P, C, F, H, W]
        pt, ph, pw = cfg.patch
        C, H, W = lat.shape[1], lat.shape[3], lat.shape[4]
        x = lat.reshape(P, C, Fr, H // ph, ph, W // pw, pw).permute(0, 2, 3, 5, 1, 4, 6) \
            .reshape(P, Fr * L, C * ph * pw)
        x = self.patch_embedding(x)
        ctx = self.text_embedding(inputs["context"]).expand(P, -1, -1)
        temb = self.time_embedding(_sinusoidal(cfg.freq_dim, inputs["timestep"].reshape(-1))
                                   .to(x.dtype))  # [P*F, d]
        t_mod = self.time_projection(temb).view(P, Fr, 6, d)
        kb = self.keyboard_embedding(inputs["keyboard"])  # [P, F*kb_rows, d]
        mouse = inputs["mouse"].reshape(P, Fr, cfg.kb_rows * cfg.mouse_dim)
        mouse = mouse[:, :, None, :].expand(P, Fr, L, -1).reshape(P, Fr * L, -1)
        x_hub = self.hub_embedding[None].expand(Fr, -1, -1).reshape(1, Fr * cfg.hub_per_frame, d)
        for i, blk in enumerate(self.blocks):
            ev = None if attn_events is None else attn_events[i]
            x, x_hub = blk(x, x_hub, ctx, mouse, kb, t_mod, consts["freqs"], consts["mask"],
                           consts["cam"], consts["frame_mask"], consts["kb_mask"],
                           consts["rope_f"], events=ev)
        hm = (self.head_modulation + temb.view(P, Fr, 1, d)).unbind(2)
        shift, scale = (_frame_mod(m_, L) for m_ in hm)
        return self.head(_modulate(self.head_norm(x), shift, scale))


def dit_inputs(cfg: DiTConfig, device, seed: int = 0):
    """Seeded inputs of configuration 3: latents ``[P,48,F,22,40]``, text
    context ``[1,512,4096]`` ~ N(0,1), timestep 500 for every frame, keyboard
    ``[P, F*12, 23]``, mouse ``[P, F*12, 2]``, camera12 ``[P, F, 12]``."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    P, Fr = cfg.players, cfg.frames
    bf = torch.bfloat16

    def rn(*s):
        return torch.randn(*s, generator=g).to(device, bf)

    return {"latents": rn(P, cfg.in_dim, Fr, cfg.height, cfg.width),
            "context": rn(1, cfg.text_len, cfg.text_dim),
            "timestep": torch.full((P, Fr), 500.0, device=device),
            "keyboard": rn(P, Fr * cfg.kb_rows, cfg.kb_dim),
            "mouse": rn(P, Fr * cfg.kb_rows, cfg.mouse_dim),
            "camera": rn(P, Fr, cfg.cam_dim)}


def init_weights(model: nn.Module, std: float = 0.02, seed: int = 0):
    """N(0, std) weights (LayerNorm / RMSNorm weights 1, biases 0), generated
    on the model's device."""
    gen = torch.Generator(device=next(model.parameters()).device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() >= 2 and "modulation" not in name and "hub_embedding" not in name:
                p.normal_(0.0, std, generator=gen)
            elif name.endswith("bias"):
                p.zero_()

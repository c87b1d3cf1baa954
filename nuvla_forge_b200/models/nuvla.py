"""nuVLA-shaped planner: multi-view/multi-frame ViT -> (fusion | VLM backbone) -> DiT + reasoning head.

Parity: nuvla_forge/model/nuvla.py:26-170. ``NuVLAConfig()`` with no
arguments builds the reference's default 77.3 M model with the same
``state_dict`` keys (encoder, fusion, scene_queries, scene_attn, dit,
text_embed, text_blocks, lm_head).

``NuVLAConfig.preset(name)`` builds the BASELINE configurations, which need
what the reference cannot express (its gaps are listed beside each field):

* ``tiny``: 6 views x 2 frames, 128 px, patch 16, ViT d=256 x 4; text backbone
  d=256 x 4, SwiGLU 704; 32 instruction + 64 reasoning tokens; DiT d=256 x 4;
  8 waypoints x (x, y, heading); t ~ U[0, 1000).
* ``1b``: 448 px, patch 14, ViT d=1024 x 24 (16 heads), tokens pooled 2x2 to
  256 per image; backbone d=2048 x 16, GQA 16q/8kv, SwiGLU 5632; 64 + 256
  text tokens; DiT d=1024 x 12; 16 waypoints x 3.
* ``3b``: as ``1b`` with backbone d=3072 x 28, GQA 24q/8kv, SwiGLU 8192 and
  DiT d=1536 x 16.

In the BASELINE layout the image tokens (after pooling and a projection to
the backbone width) and the text tokens form one causal sequence through the
backbone; the DiT cross-attends to the backbone hidden states and the
reasoning head predicts the next text token. In the reference layout a
bidirectional text branch runs over [32 scene tokens ; text] and the DiT
cross-attends to the scene tokens (nuvla_forge/model/nuvla.py:126-165).

Images enter as uint8 HWC frames [B, V*F, H, W, 3] (normalised and patchified
on the device by one kernel) or, for API parity, as normalised float
[B, V*F, 3, H, W].
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, replace

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import chunked_cross_entropy, patchify_images
from ..ops import attention as attention_op
from ..ops.image import patch_kpad
from .dit import TrajectoryDiT
from .layers import RMSNorm, TransformerBlock, _linear, linear, run_blocks


@dataclass
class NuVLAConfig:
    image_size: int = 224
    patch_size: int = 16
    n_views: int = 6
    n_frames: int = 1                # ref: frames must be folded into n_views
    vision_dim: int = 384
    vision_depth: int = 6
    vision_heads: int = 6
    vision_mlp_ratio: float = 4.0
    pool: int = 1                    # ref: no pooling
    fusion_depth: int = 4
    n_scene_queries: int = 32
    text_dim: int = 0                # 0 -> vision_dim (ref: text branch at vision width)
    text_depth: int = 2
    text_heads: int = 0              # 0 -> vision_heads
    text_kv_heads: int = 0           # 0 -> MHA (ref: no GQA)
    text_ffn: int = 0                # 0 -> 4 * text_dim
    backbone_over_images: bool = False   # BASELINE layout (causal backbone over [images ; text])
    dit_dim: int = 0                 # 0 -> vision_dim
    dit_depth: int = 6
    dit_heads: int = 0               # 0 -> vision_heads
    horizon: int = 6
    traj_dim: int = 2                # ref: (x, y) only
    t_max: float = 1.0               # ref: t ~ U(0, 1)
    vocab_size: int = 32000
    max_text_len: int = 64
    n_instruction: int = 0
    n_reasoning: int = 0
    ce_chunk_size: int = 1024
    fused: bool = True

    @property
    def n_images(self) -> int:
        return self.n_views * self.n_frames

    @property
    def tokens_per_view(self) -> int:
        return (self.image_size // self.patch_size) ** 2

    @property
    def pooled_tokens(self) -> int:
        g = self.image_size // self.patch_size
        return (g // self.pool) ** 2

    @property
    def t_dim(self) -> int:
        return self.text_dim or self.vision_dim

    @property
    def text_len(self) -> int:
        return (self.n_instruction + self.n_reasoning) or self.max_text_len

    @staticmethod
    def preset(name: str, **overrides) -> "NuVLAConfig":
        base = {
            "ref": {},
            "tiny": dict(image_size=128, patch_size=16, n_views=6, n_frames=2, vision_dim=256, vision_depth=4,
                         vision_heads=4, pool=1, fusion_depth=0, n_scene_queries=0, text_dim=256, text_depth=4,
                         text_heads=4, text_kv_heads=4, text_ffn=704, backbone_over_images=True, dit_dim=256,
                         dit_depth=4, dit_heads=4, horizon=8, traj_dim=3, t_max=1000.0, n_instruction=32,
                         n_reasoning=64),
            "1b": dict(image_size=448, patch_size=14, n_views=6, n_frames=2, vision_dim=1024, vision_depth=24,
                       vision_heads=16, pool=2, fusion_depth=0, n_scene_queries=0, text_dim=2048, text_depth=16,
                       text_heads=16, text_kv_heads=8, text_ffn=5632, backbone_over_images=True, dit_dim=1024,
                       dit_depth=12, dit_heads=16, horizon=16, traj_dim=3, t_max=1000.0, n_instruction=64,
                       n_reasoning=256),
            "3b": dict(image_size=448, patch_size=14, n_views=6, n_frames=2, vision_dim=1024, vision_depth=24,
                       vision_heads=16, pool=2, fusion_depth=0, n_scene_queries=0, text_dim=3072, text_depth=28,
                       text_heads=24, text_kv_heads=8, text_ffn=8192, backbone_over_images=True, dit_dim=1536,
                       dit_depth=16, dit_heads=16, horizon=16, traj_dim=3, t_max=1000.0, n_instruction=64,
                       n_reasoning=256),
        }
        if name not in base:
            raise KeyError(f"unknown preset {name!r}; have {sorted(base)}")
        return replace(NuVLAConfig(), **{**base[name], **overrides})

    def to_dict(self) -> dict:
        return asdict(self)


class MultiViewEncoder(nn.Module):
    """Shared ViT over all views and frames with learned camera (and frame) embeddings.

    Parity: nuvla_forge/model/nuvla.py:62-94. The patch embedding keeps the
    Conv2d parameter shape ([D, 3, p, p] + bias, key ``patch.weight``) but runs
    as a GEMM over patch rows produced by the fused uint8 -> bf16 patchify kernel.
    """

    def __init__(self, cfg: NuVLAConfig):
        super().__init__()
        self.cfg = cfg
        d = cfg.vision_dim
        p = cfg.patch_size
        self.patch = nn.Conv2d(3, d, p, p)
        self.pos = nn.Parameter(torch.zeros(1, cfg.tokens_per_view, d))
        self.cam_embed = nn.Parameter(torch.zeros(cfg.n_views, d))
        nn.init.normal_(self.pos, std=0.02)
        nn.init.normal_(self.cam_embed, std=0.02)
        if cfg.n_frames > 1:
            self.frame_embed = nn.Parameter(torch.zeros(cfg.n_frames, d))
            nn.init.normal_(self.frame_embed, std=0.02)
        else:
            self.frame_embed = None
        self.blocks = nn.ModuleList([
            TransformerBlock(d, cfg.vision_heads, cfg.fused, ffn=int(d * cfg.vision_mlp_ratio))
            for _ in range(cfg.vision_depth)
        ])
        self.norm = RMSNorm(d, fused=cfg.fused)

    def image_embed(self) -> torch.Tensor:
        """[V*F, D] embedding per image index (view-major, frame-minor)."""
        e = self.cam_embed
        if self.frame_embed is not None:
            e = (self.cam_embed[:, None, :] + self.frame_embed[None, :, :]).reshape(-1, e.shape[-1])
        return e

    def embed_patches(self, images: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        p = cfg.patch_size
        d = cfg.vision_dim
        wdt = self.patch.weight.dtype
        if images.dtype == torch.uint8:  # [B, NI, H, W, 3]
            b, ni, H, W, _ = images.shape
            kpad = patch_kpad(p)
            rows = patchify_images(images.reshape(b * ni, H, W, 3), p, dtype=wdt, kpad=kpad,
                                   force_reference=not cfg.fused)
            w = self.patch.weight.reshape(d, -1)
            if kpad != w.shape[1]:
                w = F.pad(w, (0, kpad - w.shape[1]))
            x = linear(rows, w, self.patch.bias)  # [B*NI, P, D]
        else:  # normalised float [B, NI, 3, H, W]
            b, ni = images.shape[:2]
            x = self.patch(images.flatten(0, 1).to(wdt))
            x = x.flatten(2).transpose(1, 2)
        return x, b, ni

    def forward(self, images):
        """images -> [B, NI * P, D] (all views and frames, view-major)."""
        x, b, ni = self.embed_patches(images)
        x = x + self.pos
        x = x + self.image_embed().repeat(b, 1).unsqueeze(1)
        x = run_blocks(self.blocks, x, self.norm)
        return x.reshape(b, ni * x.shape[1], x.shape[2])


class SceneQueryPool(nn.Module):
    """32 learned queries attend over all view tokens (nn.MultiheadAttention parameter layout).

    Parity: nuvla_forge/model/nuvla.py:107-112,126-132; keys ``in_proj_weight``,
    ``in_proj_bias``, ``out_proj.weight``, ``out_proj.bias``.
    """

    def __init__(self, dim: int, heads: int, fused: bool = True):
        super().__init__()
        self.heads = heads
        self.fused = fused
        self.in_proj_weight = nn.Parameter(torch.empty(3 * dim, dim))
        self.in_proj_bias = nn.Parameter(torch.zeros(3 * dim))
        self.out_proj = nn.Linear(dim, dim)
        nn.init.xavier_uniform_(self.in_proj_weight)
        nn.init.zeros_(self.out_proj.bias)

    def forward(self, q, x):
        b, s, d = q.shape
        L = x.shape[1]
        h = self.heads
        dh = d // h
        wq, wkv = self.in_proj_weight[:d], self.in_proj_weight[d:]
        bq, bkv = self.in_proj_bias[:d], self.in_proj_bias[d:]
        qq = linear(q, wq, bq).view(b, s, h, dh)
        kv = linear(x, wkv, bkv).view(b, L, 2 * h, dh)
        k, v = kv.split([h, h], dim=2)
        o = attention_op(qq, k, v, causal=False, force_reference=not self.fused).reshape(b, s, d)
        return linear(o, self.out_proj.weight, self.out_proj.bias)


class NuVLA(nn.Module):
    def __init__(self, cfg: NuVLAConfig | None = None):
        super().__init__()
        self.cfg = cfg = cfg or NuVLAConfig()
        dv = cfg.vision_dim
        dt = cfg.t_dim
        dd = cfg.dit_dim or dv
        self.encoder = MultiViewEncoder(cfg)
        self.fusion = nn.ModuleList([TransformerBlock(dv, cfg.vision_heads, cfg.fused)
                                     for _ in range(cfg.fusion_depth)])
        if cfg.n_scene_queries > 0:
            self.scene_queries = nn.Parameter(torch.zeros(1, cfg.n_scene_queries, dv))
            nn.init.normal_(self.scene_queries, std=0.02)
            self.scene_attn = SceneQueryPool(dv, cfg.vision_heads, cfg.fused)
        if cfg.backbone_over_images:
            self.vision_proj = nn.Linear(dv, dt, bias=False)
            self.text_pos = nn.Parameter(torch.zeros(1, cfg.text_len, dt))
            nn.init.normal_(self.text_pos, std=0.02)
            ctx_dim = dt
        else:
            ctx_dim = dv
        self.dit = TrajectoryDiT(dim=dd, depth=cfg.dit_depth, n_heads=cfg.dit_heads or cfg.vision_heads,
                                 horizon=cfg.horizon, fused=cfg.fused, traj_dim=cfg.traj_dim, ctx_dim=ctx_dim,
                                 t_max=cfg.t_max)
        self.text_embed = nn.Embedding(cfg.vocab_size, dt)
        th = cfg.text_heads or cfg.vision_heads
        self.text_blocks = nn.ModuleList([
            TransformerBlock(dt, th, cfg.fused, kv_heads=cfg.text_kv_heads or None, ffn=cfg.text_ffn or None,
                             causal=cfg.backbone_over_images)
            for _ in range(cfg.text_depth)
        ])
        if cfg.backbone_over_images:
            self.text_norm = RMSNorm(dt, fused=cfg.fused)
        self.lm_head = nn.Parameter(torch.empty(cfg.vocab_size, dt))
        nn.init.normal_(self.lm_head, std=0.02)

    # -- reference layout -------------------------------------------------
    def encode_scene(self, images):
        x = self.encoder(images)
        b = x.shape[0]
        x = run_blocks(self.fusion, x)
        if self.cfg.n_scene_queries > 0:
            return self.scene_attn(self.scene_queries.expand(b, -1, -1), x)
        return x

    # -- BASELINE layout --------------------------------------------------
    def image_tokens(self, images):
        cfg = self.cfg
        x = self.encoder(images)                     # [B, NI*P, Dv]
        b, ni, P, d = x.shape[0], cfg.n_images, cfg.tokens_per_view, x.shape[-1]
        if cfg.pool > 1:
            g = int(round(P ** 0.5))
            k = cfg.pool
            x = x.view(b * ni, g // k, k, g // k, k, d).mean(dim=(2, 4))
        x = x.reshape(b, -1, d)
        return linear(x, self.vision_proj.weight)  # [B, NI*Pp, Dt]

    def forward(self, images, trajectory=None, text_tokens=None, text_targets=None):
        """Joint objective: flow-matching plan loss + reasoning cross entropy (summed)."""
        cfg = self.cfg
        out = {}
        losses = []
        if cfg.backbone_over_images:
            img = self.image_tokens(images)
            n_img = img.shape[1]
            if text_tokens is not None:
                txt = self.text_embed(text_tokens) + self.text_pos[:, : text_tokens.shape[1]]
                h = torch.cat([img, txt.to(img.dtype)], dim=1)
            else:
                h = img
            h = run_blocks(self.text_blocks, h, self.text_norm)
            context = h
            text_h = h[:, n_img:]
        else:
            scene = self.encode_scene(images)
            context = scene
            text_h = None
            if text_tokens is not None:
                t = self.text_embed(text_tokens)
                h = torch.cat([scene, t.to(scene.dtype)], dim=1)
                h = run_blocks(self.text_blocks, h)
                text_h = h[:, scene.shape[1]:]
        if trajectory is not None:
            plan = self.dit.flow_loss(trajectory, context)
            out["plan_loss"] = plan.detach()
            losses.append(plan)
        if text_h is not None and text_targets is not None:
            reason = chunked_cross_entropy(text_h.reshape(-1, text_h.shape[-1]), self.lm_head,
                                           text_targets.reshape(-1), chunk_size=cfg.ce_chunk_size,
                                           force_reference=not cfg.fused)
            out["reason_loss"] = reason.detach()
            losses.append(reason)
        total = losses[0] if losses else context.new_zeros((), dtype=torch.float32)
        for l in losses[1:]:
            total = total + l
        out["loss"] = total
        return out

    @torch.no_grad()
    def context(self, images, text_tokens=None):
        """The states the DiT cross-attends to (backbone output over image and instruction tokens)."""
        cfg = self.cfg
        if cfg.backbone_over_images:
            img = self.image_tokens(images)
            h = img
            if text_tokens is not None:
                txt = self.text_embed(text_tokens) + self.text_pos[:, : text_tokens.shape[1]]
                h = torch.cat([img, txt.to(img.dtype)], dim=1)
            return run_blocks(self.text_blocks, h, self.text_norm)
        return self.encode_scene(images)

    @torch.no_grad()
    def plan(self, images, text_tokens=None, steps: int = 10, z0: torch.Tensor | None = None):
        """Sample waypoints [B, horizon, traj_dim] by Euler integration of the DiT's velocity."""
        return self.dit.sample(self.context(images, text_tokens), steps=steps, z0=z0)

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())


__all__ = ["MultiViewEncoder", "NuVLA", "NuVLAConfig", "SceneQueryPool", "_linear"]

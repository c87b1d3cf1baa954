"""Trajectory DiT with adaLN-Zero conditioning, trained by rectified flow.

Parity: nuvla_forge/model/dit.py:113-230 (DiTBlock, TrajectoryDiT, flow_loss,
sample). Same parameters and the same function; the fused path differs in
how the seams are scheduled:

* Every seam "gated residual add -> RMSNorm -> adaLN modulate" is ONE native
  kernel (ops.fused_adaln_residual_rmsnorm), including the seam that crosses
  a block boundary: a block hands its un-added, gated MLP output to the next
  block (or to the final norm), which folds ``x + gate2 * mlp`` into its own
  norm1 + modulate. The reference left that add eager
  (nuvla_forge/model/dit.py:169).
* The cross-attention residual (gate 1) is read by the output-projection GEMM.

Generalisations for the BASELINE configs: waypoints of any width (x, y,
heading), a context of a different width than the DiT (cross-attention keys
and values come from backbone hidden states), and a diffusion time range
``t_max`` (t ~ U[0, t_max) feeds the sinusoid; the interpolation uses t / t_max).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import fused_adaln_residual_rmsnorm
from .layers import Attention, RMSNorm, SwiGLUMLP, TimestepEmbedder, checkpointed, linear, modulate


class DiTBlock(nn.Module):
    def __init__(self, dim: int, n_heads: int, mlp_ratio: float = 4.0, fused: bool = True,
                 ctx_dim: int | None = None):
        super().__init__()
        self.dim = dim
        self.fused = fused
        self.norm1 = RMSNorm(dim, fused=fused)
        self.norm2 = RMSNorm(dim, fused=fused)
        self.attn = Attention(dim, n_heads, fused=fused)
        self.cross = Attention(dim, n_heads, ctx_dim=ctx_dim, fused=fused)
        self.norm_cross = RMSNorm(dim, fused=fused)
        self.mlp = SwiGLUMLP(dim, int(dim * mlp_ratio), fused=fused)
        self.cond = nn.Sequential(nn.SiLU(), nn.Linear(dim, 6 * dim, bias=True))
        # adaLN-Zero: every block starts as the identity on the residual stream.
        nn.init.zeros_(self.cond[1].weight)
        nn.init.zeros_(self.cond[1].bias)
        self.grad_checkpoint = False  # recompute the block in backward (models/layers.checkpointed)

    def _cond(self, c):
        lin = self.cond[1]
        return linear(F.silu(c), lin.weight, lin.bias)

    def forward_chain(self, x, c, context, pending=None):
        """Fused path. ``pending`` = (y, gate): the previous block's gated branch
        output not yet added to x. Returns (x, (mlp_out, gate2))."""
        return checkpointed(self, self._chain, x, c, context, pending)

    def _chain(self, x, c, context, pending):
        b, t, _ = x.shape
        shift1, scale1, gate1, shift2, scale2, gate2 = self._cond(c).chunk(6, dim=-1)
        if pending is None:
            h = self.norm1(x, scale=scale1, shift=shift1, tokens_per_sample=t)
        else:
            y, g = pending
            x, h = fused_adaln_residual_rmsnorm(x, y, g, self.norm1.weight, scale1, shift1, t, self.norm1.eps)
        a = self.attn(h)
        x, h = fused_adaln_residual_rmsnorm(x, a, gate1, self.norm_cross.weight, None, None, t,
                                            self.norm_cross.eps)
        x = self.cross(h, context, residual=x)
        h = self.norm2(x, scale=scale2, shift=shift2, tokens_per_sample=t)
        return x, (self.mlp(h), gate2)

    def forward(self, x, c, context):
        if self.fused:
            x, (m, g) = self.forward_chain(x, c, context)
            return x + g.unsqueeze(1) * m
        return checkpointed(self, self._forward_unfused, x, c, context)

    def _forward_unfused(self, x, c, context):
        shift1, scale1, gate1, shift2, scale2, gate2 = self._cond(c).chunk(6, dim=-1)
        x = x + gate1.unsqueeze(1) * self.attn(modulate(self.norm1(x), shift1, scale1))
        x = x + self.cross(self.norm_cross(x), context)
        return x + gate2.unsqueeze(1) * self.mlp(modulate(self.norm2(x), shift2, scale2))


class TrajectoryDiT(nn.Module):
    """Denoises a [B, horizon, traj_dim] ego trajectory conditioned on context tokens."""

    def __init__(self, dim: int = 384, depth: int = 6, n_heads: int = 6, horizon: int = 6, fused: bool = True,
                 traj_dim: int = 2, ctx_dim: int | None = None, t_max: float = 1.0):
        super().__init__()
        self.horizon = horizon
        self.traj_dim = traj_dim
        self.t_max = float(t_max)
        self.fused = fused
        ctx_dim = ctx_dim or dim
        self.in_proj = nn.Linear(traj_dim, dim)
        self.pos = nn.Parameter(torch.zeros(1, horizon, dim))
        nn.init.normal_(self.pos, std=0.02)
        self.t_embed = TimestepEmbedder(dim)
        self.scene_proj = nn.Linear(ctx_dim, dim)
        self.blocks = nn.ModuleList([DiTBlock(dim, n_heads, fused=fused, ctx_dim=ctx_dim) for _ in range(depth)])
        self.norm_out = RMSNorm(dim, fused=fused)
        self.out = nn.Linear(dim, traj_dim)
        nn.init.zeros_(self.out.weight)
        nn.init.zeros_(self.out.bias)

    def forward(self, z_t, t, context):
        wdt = self.in_proj.weight.dtype
        x = linear(z_t.to(wdt), self.in_proj.weight, self.in_proj.bias) + self.pos
        c = self.t_embed(t) + linear(context.mean(dim=1), self.scene_proj.weight, self.scene_proj.bias)
        if self.fused:
            pending = None
            for blk in self.blocks:
                x, pending = blk.forward_chain(x, c, context, pending)
            if pending is None:
                h = self.norm_out(x)
            else:
                m, g = pending
                _, h = fused_adaln_residual_rmsnorm(x, m, g, self.norm_out.weight, None, None, x.shape[1],
                                                    self.norm_out.eps)
        else:
            for blk in self.blocks:
                x = blk(x, c, context)
            h = self.norm_out(x)
        return linear(h, self.out.weight, self.out.bias)

    def flow_loss(self, trajectory, context):
        """Rectified flow: z_t = (1 - s) noise + s traj with s = t / t_max; regress traj - noise."""
        b = trajectory.shape[0]
        traj = trajectory.to(torch.float32)
        noise = torch.randn_like(traj)
        t = torch.rand(b, device=traj.device) * self.t_max
        s = (t / self.t_max)[:, None, None]
        z_t = (1 - s) * noise + s * traj
        pred = self(z_t, t, context)
        return F.mse_loss(pred.float(), traj - noise)

    @torch.no_grad()
    def sample(self, context, steps: int = 10, z0: torch.Tensor | None = None):
        """Euler integration of the learned velocity from noise (s=0) to a trajectory (s=1).

        ``z0`` (optional) is the starting noise [B, horizon, traj_dim]; drawn here when omitted.
        """
        b = context.shape[0]
        z = z0.float() if z0 is not None else torch.randn(b, self.horizon, self.traj_dim, device=context.device,
                                                          dtype=torch.float32)
        ds = 1.0 / steps
        for i in range(steps):
            t = torch.full((b,), i * ds * self.t_max, device=z.device)
            z = z + self(z, t, context).float() * ds
        return z

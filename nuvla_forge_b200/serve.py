"""Planning (inference) with the DiT sampling loop captured in one CUDA graph.

At serving batch sizes the sampler is launch-bound: every Euler step runs the
whole DiT (a few hundred small kernels) on a [B, horizon] trajectory. The
``GraphedPlanner`` captures all ``steps`` Euler steps for a fixed batch size
and context length once (after a warm-up on a side stream, which also
initialises every kernel's lazily created state), and then serves each
request with two copies into static buffers and one graph replay.

    planner = GraphedPlanner(model, batch_size=8, context_len=L, steps=10)
    waypoints = planner(context)          # context: model.context(images, text_tokens)

On CPU (or with ``graph=False``) it runs the same sampler eagerly.
The reference has no inference path beyond ``TrajectoryDiT.sample``
(nuvla_forge/model/dit.py:221-230, never called in its repository).
"""

from __future__ import annotations

import torch

from .models.nuvla import NuVLA


class GraphedPlanner:
    def __init__(self, model: NuVLA, batch_size: int, context_len: int, steps: int = 10, graph: bool = True,
                 warmup: int = 2):
        self.model = model
        self.dit = model.dit
        self.steps = steps
        p = next(model.parameters())
        self.device = p.device
        d_ctx = self._context_dim(model)
        self.ctx = torch.zeros(batch_size, context_len, d_ctx, device=self.device, dtype=p.dtype)
        self.z0 = torch.zeros(batch_size, self.dit.horizon, self.dit.traj_dim, device=self.device)
        self.out = None
        self.graph = None
        if graph and self.device.type == "cuda":
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side), torch.no_grad():
                for _ in range(warmup):
                    self.dit.sample(self.ctx, self.steps, z0=self.z0)
            torch.cuda.current_stream(self.device).wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g), torch.no_grad():
                self.out = self.dit.sample(self.ctx, self.steps, z0=self.z0)
            self.graph = g

    @staticmethod
    def _context_dim(model: NuVLA) -> int:
        cfg = model.cfg
        return cfg.t_dim if cfg.backbone_over_images else cfg.vision_dim

    @torch.no_grad()
    def __call__(self, context: torch.Tensor, z0: torch.Tensor | None = None) -> torch.Tensor:
        """Waypoints [B, horizon, traj_dim] for ``context`` [B, context_len, D] (fresh noise unless ``z0``)."""
        if context.shape != self.ctx.shape:
            raise ValueError(f"planner was built for context {tuple(self.ctx.shape)}, got {tuple(context.shape)}")
        self.ctx.copy_(context)
        if z0 is not None:
            self.z0.copy_(z0)
        else:
            self.z0.normal_()
        if self.graph is None:
            return self.dit.sample(self.ctx, self.steps, z0=self.z0)
        self.graph.replay()
        return self.out.clone()

"""Flat parameter / gradient storage.

All trainable parameters of a module are re-homed as views of ONE contiguous
low-precision buffer (what the model computes with) and get an fp32 master
copy and an fp32 gradient accumulator in matching flat buffers. Segments are
8-element aligned so every vector kernel can run over any segment or over the
whole space in one launch. Parameters are laid out in reverse registration
order, which approximates the order autograd produces their gradients, so a
contiguous range of the space fills up early in backward and can be reduced
while backward continues.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

ALIGN = 8


def _round(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


@dataclass
class Segment:
    name: str
    param: nn.Parameter
    start: int
    numel: int
    shape: torch.Size


class FlatParamSpace:
    def __init__(self, module: nn.Module, param_dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | None = None, align: int = ALIGN):
        named = [(n, p) for n, p in module.named_parameters() if p.requires_grad]
        named.reverse()
        dev = device or named[0][1].device
        self.device = dev
        self.param_dtype = param_dtype
        self.segments: list[Segment] = []
        off = 0
        for n, p in named:
            self.segments.append(Segment(n, p, off, p.numel(), p.shape))
            off += _round(p.numel(), align)
        self.align = align
        self.numel = _round(off, align)
        self.params = torch.zeros(self.numel, dtype=param_dtype, device=dev)
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        self.grads = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        with torch.no_grad():
            for s in self.segments:
                src = s.param.detach().reshape(-1)
                self.master[s.start: s.start + s.numel].copy_(src.to(torch.float32))
                self.params[s.start: s.start + s.numel].copy_(src.to(param_dtype))
                s.param.data = self.params[s.start: s.start + s.numel].view(s.shape)
                s.param.main_grad = self.grads[s.start: s.start + s.numel].view(s.shape)
        self.by_param = {id(s.param): s for s in self.segments}

    def segment(self, p: nn.Parameter) -> Segment:
        return self.by_param[id(p)]

    def sync_params_from_master(self) -> None:
        with torch.no_grad():
            self.params.copy_(self.master.to(self.param_dtype))

    def master_state_dict(self, prefix_map=None) -> dict[str, torch.Tensor]:
        """fp32 copies of every parameter under its module name."""
        out = {}
        for s in self.segments:
            out[s.name] = self.master[s.start: s.start + s.numel].view(s.shape).clone()
        return out

    def load_master(self, named: dict[str, torch.Tensor]) -> None:
        with torch.no_grad():
            for s in self.segments:
                if s.name in named:
                    self.master[s.start: s.start + s.numel].copy_(named[s.name].reshape(-1).to(torch.float32))
        self.sync_params_from_master()

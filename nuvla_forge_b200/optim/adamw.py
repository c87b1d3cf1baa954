"""AdamW over a flat parameter space, with global-norm clipping that never syncs the host.

Parity: the reference steps ``torch.optim.AdamW(lr, weight_decay=0.01,
fused=True)`` after ``clip_grad_norm_(params, 1.0)`` (nuvla_forge/train.py:
170-173, 228-230). Here the norm is one deterministic reduction kernel over the
flat fp32 gradient buffer whose result stays on the device, and the update is
one launch over the flat fp32 master buffer that also writes the bf16 compute
copy (csrc/optim.cu). On CPU the same math runs as torch ops.
"""

from __future__ import annotations

import math

import torch

from .. import _native as nat


class FlatAdamW:
    def __init__(self, space, lr: float = 3e-4, betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, max_grad_norm: float = 1.0, ddp=None, grads: torch.Tensor | None = None,
                 master: torch.Tensor | None = None, params: torch.Tensor | None = None,
                 norm_allreduce=None, params_ptr: int | None = None, after_step=None):
        self.space = space
        self.master = master if master is not None else space.master
        self.grads = grads if grads is not None else space.grads
        self.params = params if params is not None else space.params
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_grad_norm = max_grad_norm
        self.ddp = ddp
        self.norm_allreduce = norm_allreduce   # FSDP: sums the norm^2 over ranks on the device
        self.params_ptr = params_ptr           # raw bf16 destination (FSDP: the peer-mapped shard region)
        self.after_step = after_step
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.step_count = 0
        dev = self.master.device
        self.native = dev.type == "cuda" and nat.HAS_NATIVE
        self.norm2 = torch.zeros(1, dtype=torch.float32, device=dev)
        if self.native:
            self._partials = torch.empty(int(nat.lib().nfb_sumsq_slots()), dtype=torch.float32, device=dev)
            self._ticket = torch.zeros(1, dtype=torch.int32, device=dev)

    # ------------------------------------------------------------------
    def compute_norm2(self) -> torch.Tensor:
        if self.native:
            nat.call("nfb_sumsq", 0, nat.ptr(self.grads), self.grads.numel(), 1.0, nat.ptr(self._partials),
                     nat.ptr(self._ticket), nat.ptr(self.norm2), 0, nat.stream(self.grads.device))
        else:
            self.norm2.copy_(self.grads.double().square().sum().float().view(1))
        if self.norm_allreduce is not None:
            self.norm_allreduce(self.norm2)
        return self.norm2

    def grad_norm(self) -> torch.Tensor:
        """Global gradient norm of the last step (device scalar; no host sync)."""
        return self.norm2.sqrt()

    def step(self) -> None:
        self.step_count += 1
        owner = getattr(self, "fused_owner", None)
        if owner is not None and owner.take_fused_step():
            # FSDP already applied this step inside each unit's reduce-scatter
            if self.after_step is not None:
                self.after_step()
            return
        clip = self.max_grad_norm is not None and self.max_grad_norm > 0
        if clip:
            take = getattr(owner, "take_norm2", None) if owner is not None else None
            if take is not None and take():
                # the reduce-scatters already summed this rank's squared gradient shard (clip phase 1);
                # only the sum over ranks remains
                if self.norm_allreduce is not None:
                    self.norm_allreduce(self.norm2)
            else:
                self.compute_norm2()
        b1, b2 = self.betas
        if self.native:
            import ctypes

            lp = self.params if (self.params is not None and self.params.dtype == torch.bfloat16) else None
            lp_ptr = ctypes.c_void_p(self.params_ptr) if self.params_ptr is not None else nat.ptr(lp)
            nat.call("nfb_adamw_flat", nat.ptr(self.master), nat.ptr(self.grads), nat.ptr(self.m), nat.ptr(self.v),
                     lp_ptr, self.master.numel(), self.lr, b1, b2, self.eps, self.weight_decay,
                     self.step_count, 1.0, nat.ptr(self.norm2) if clip else nat.ptr(None),
                     float(self.max_grad_norm if clip else 0.0), nat.stream(self.master.device))
            if (self.params_ptr is None and lp is None and self.params is not None
                    and self.params.data_ptr() != self.master.data_ptr()):
                self.params.copy_(self.master)
            if self.after_step is not None:
                self.after_step()
            return
        with torch.no_grad():
            g = self.grads
            if clip:
                coef = torch.clamp(self.max_grad_norm / (self.norm2.sqrt() + 1e-6), max=1.0)
                g = g * coef
            p = self.master
            p.mul_(1 - self.lr * self.weight_decay)
            self.m.mul_(b1).add_(g, alpha=1 - b1)
            self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
            bc1 = 1 - b1 ** self.step_count
            bc2 = 1 - b2 ** self.step_count
            denom = (self.v.sqrt() / math.sqrt(bc2)).add_(self.eps)
            p.addcdiv_(self.m, denom, value=-self.lr / bc1)
            if self.params is not None and self.params.data_ptr() != p.data_ptr():
                self.params.copy_(p.to(self.params.dtype))
        if self.after_step is not None:
            self.after_step()

    def zero_grad(self, set_to_none: bool = True) -> None:
        if self.ddp is not None:
            self.ddp.zero_grad()
        else:
            self.grads.zero_()

    # ------------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"step": self.step_count, "lr": self.lr, "betas": self.betas, "eps": self.eps,
                "weight_decay": self.weight_decay, "exp_avg": self.m.detach().cpu(),
                "exp_avg_sq": self.v.detach().cpu()}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.lr = sd.get("lr", self.lr)
        self.m.copy_(sd["exp_avg"].to(self.m.device))
        self.v.copy_(sd["exp_avg_sq"].to(self.v.device))

"""Transformer building blocks shared by the vision encoder, the backbone and the DiT.

Parameter names follow the reference so ``state_dict`` keys match
(nuvla_forge/model/dit.py:34-110, nuvla_forge/model/nuvla.py:47-59):
``norm1/norm2.weight``, ``attn.qkv.weight``, ``attn.proj.weight``,
``mlp.w_gate.weight``, ``mlp.w_up.weight``, ``mlp.w_down.weight``.

Compute differs from the reference where it saves memory traffic, never in
the function computed:

* Every linear layer runs its forward, input-gradient and weight-gradient
  GEMMs on the native CTA-pair tcgen05 kernel (``ops.linear``); residual adds
  are fused into the output-projection GEMM epilogue, and the following
  RMSNorm is one native kernel.
* The SwiGLU gate and up projections are one GEMM over a packed [2F, D]
  weight whose backward is one input-gradient GEMM; ``state_dict`` still
  exposes ``w_gate.weight`` and ``w_up.weight`` (split on save, joined on load).
* Attention runs on the projection-native [B, S, H, D] layout (no permutes)
  and supports grouped-query attention (``kv_heads < heads``) and a causal
  mask, which the BASELINE backbone configs need.
"""

from __future__ import annotations

import math

import torch
import torch.utils.checkpoint
import torch.nn.functional as F
from torch import nn

from ..ops import add_rmsnorm
from ..ops import attention as attention_op
from ..ops import linear as linear_op
from ..ops import rmsnorm as rmsnorm_op
from ..ops import fused_swiglu, swiglu_packed
from ..ops.reference import swiglu_ref


# A parameter owner (the FSDP runtime) that deferred gathering a unit's
# parameters to the unit's first linear layer; it returns that layer's output
# (computed by the all-gather-fused GEMM) or None to let F.linear run.
_pending_consumer = None


def set_pending_consumer(fn) -> None:
    """Register (or clear, with None) the callable that gets the next linear() call."""
    global _pending_consumer
    _pending_consumer = fn


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """x @ w.T (+ b) on the native GEMM, unless a pending parameter consumer computes it first."""
    fn = _pending_consumer
    if fn is not None:
        y = fn(x, w, b)
        if y is not None:
            return y
    return linear_op.linear(x, w, b)


def _linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
            residual: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w.T (+ b) (+ residual), with the residual read by the GEMM epilogue."""
    if residual is None:
        return linear(x, w, b)
    return linear_op.linear(x, w, b, residual=residual)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6, fused: bool = True):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps
        self.fused = fused

    def forward(self, x, scale=None, shift=None, tokens_per_sample=None):
        return rmsnorm_op(x, self.weight, self.eps, scale=scale, shift=shift,
                          tokens_per_sample=tokens_per_sample, force_reference=not self.fused)


def modulate(x, shift, scale):
    return x * (1 + scale.unsqueeze(1)) + shift.unsqueeze(1)


class TimestepEmbedder(nn.Module):
    """Sinusoidal diffusion-time embedding projected to the model width.

    Parity: nuvla_forge/model/dit.py:49-68 (freq_dim 256, Linear-SiLU-Linear).
    """

    def __init__(self, dim: int, freq_dim: int = 256):
        super().__init__()
        self.freq_dim = freq_dim
        self.mlp = nn.Sequential(nn.Linear(freq_dim, dim), nn.SiLU(), nn.Linear(dim, dim))

    def forward(self, t):
        half = self.freq_dim // 2
        k = torch.arange(half, dtype=torch.float32, device=t.device)
        freqs = torch.exp(k * (-math.log(10000.0) / half))
        ang = t.to(torch.float32)[:, None] * freqs[None, :]
        emb = torch.cat([torch.cos(ang), torch.sin(ang)], dim=-1)
        l0, l2 = self.mlp[0], self.mlp[2]
        h = F.silu(linear(emb.to(l0.weight.dtype), l0.weight, l0.bias))
        return linear(h, l2.weight, l2.bias)


class Attention(nn.Module):
    """Multi-head / grouped-query attention with a fused qkv projection.

    Self-attention uses ``qkv`` [(H + 2*Hkv) * Dh, D]. Cross-attention into a
    context of the same width slices the same weight (as the reference does,
    nuvla_forge/model/dit.py:84-90); for a context of a different width the
    module owns ``q`` [D, D] and ``kv`` [2 * Hkv * Dh, Dctx] instead.
    """

    def __init__(self, dim: int, n_heads: int, kv_heads: int | None = None, causal: bool = False,
                 ctx_dim: int | None = None, fused: bool = True):
        super().__init__()
        self.dim = dim
        self.n_heads = n_heads
        self.kv_heads = kv_heads or n_heads
        self.head_dim = dim // n_heads
        self.causal = causal
        self.fused = fused
        kvd = self.kv_heads * self.head_dim
        self.split_ctx = ctx_dim is not None and ctx_dim != dim
        if self.split_ctx:
            self.q = nn.Linear(dim, dim, bias=False)
            self.kv = nn.Linear(ctx_dim, 2 * kvd, bias=False)
        else:
            self.qkv = nn.Linear(dim, dim + 2 * kvd, bias=False)
        self.proj = nn.Linear(dim, dim, bias=False)

    def forward(self, x, context=None, residual=None):
        b, t, c = x.shape
        H, Hk, Dh = self.n_heads, self.kv_heads, self.head_dim
        if context is None:
            qkv = linear(x, self.qkv.weight).view(b, t, H + 2 * Hk, Dh)
            q, k, v = qkv.split([H, Hk, Hk], dim=2)
        else:
            s = context.shape[1]
            if self.split_ctx:
                q = linear(x, self.q.weight).view(b, t, H, Dh)
                kv = linear(context, self.kv.weight).view(b, s, 2 * Hk, Dh)
            else:
                q = linear(x, self.qkv.weight[:c]).view(b, t, H, Dh)
                kv = linear(context, self.qkv.weight[c:]).view(b, s, 2 * Hk, Dh)
            k, v = kv.split([Hk, Hk], dim=2)
        o = attention_op(q, k, v, causal=self.causal and context is None, force_reference=not self.fused)
        o = o.reshape(b, t, c)
        return _linear(o, self.proj.weight, residual=residual)


class SwiGLUMLP(nn.Module):
    """w_down(silu(w_gate x) * w_up x) with the gate/up weights packed in one tensor.

    When the hidden width is a multiple of 128 the packed weight stores gate and up rows
    interleaved in 128-row blocks, the layout of the native fused MLP (gate/up GEMM with the
    SwiGLU in its epilogue, down-projection input gradient with the SwiGLU backward in its
    epilogue); otherwise it is [gate; up]. ``state_dict`` always exposes the reference's
    ``w_gate.weight`` / ``w_up.weight`` (split on save, joined on load).
    """

    def __init__(self, dim: int, hidden: int, fused: bool = True):
        super().__init__()
        self.hidden = hidden
        self.fused = fused
        self.interleaved = hidden % 128 == 0
        self.w_gate_up = nn.Parameter(torch.empty(2 * hidden, dim))
        self.w_down = nn.Linear(hidden, dim, bias=False)
        bound = 1.0 / math.sqrt(dim)
        nn.init.uniform_(self.w_gate_up, -bound, bound)
        self._register_state_dict_hook(SwiGLUMLP._split_on_save)
        self._register_load_state_dict_pre_hook(self._join_on_load)

    @staticmethod
    def _split_on_save(module, state_dict, prefix, local_metadata):
        key = prefix + "w_gate_up"
        if key in state_dict:
            w = state_dict.pop(key)
            if module.interleaved:
                g, u = linear_op.split_gate_up_rows(w)
            else:
                g, u = w[: module.hidden], w[module.hidden:]
            state_dict[prefix + "w_gate.weight"] = g
            state_dict[prefix + "w_up.weight"] = u
        return state_dict

    def _join_on_load(self, state_dict, prefix, *args, **kwargs):
        g, u = prefix + "w_gate.weight", prefix + "w_up.weight"
        if g in state_dict and u in state_dict:
            gw, uw = state_dict.pop(g), state_dict.pop(u)
            state_dict[prefix + "w_gate_up"] = (linear_op.interleave_gate_up(gw, uw) if self.interleaved
                                                else torch.cat([gw, uw], dim=0))

    def forward(self, x, residual=None):
        w = self.w_gate_up
        if self.fused and self.interleaved and _pending_consumer is None and \
                linear_op.swiglu_supported(x, w, self.w_down.weight):
            return linear_op.swiglu_mlp(x, w, self.w_down.weight, residual)
        if self.interleaved and x.is_cuda and self.fused:
            # library-GEMM path (A/B runs, unsupported shapes): one GEMM over the [gate; up] row order
            # (a cheap weight permutation), then the packed SwiGLU kernel
            g, u = linear_op.split_gate_up_rows(w)
            act = swiglu_packed(linear(x, torch.cat([g, u], dim=0)))
            return _linear(act, self.w_down.weight, residual=residual)
        ab = linear(x, w)
        if self.interleaved:
            a, b = linear_op.split_gate_up_cols(ab)
            act = fused_swiglu(a, b) if self.fused else swiglu_ref(a, b)
        elif self.fused:
            act = swiglu_packed(ab)
        else:
            act = swiglu_ref(ab[..., : self.hidden], ab[..., self.hidden:])
        return _linear(act, self.w_down.weight, residual=residual)


def checkpointed(block: nn.Module, fn, *args):
    """``fn(*args)``, recomputed in backward when ``block.grad_checkpoint`` is set and autograd is
    recording: only the block's inputs stay alive between forward and backward
    (torch.utils.checkpoint, non-reentrant, RNG state preserved)."""
    if getattr(block, "grad_checkpoint", False) and torch.is_grad_enabled():
        return torch.utils.checkpoint.checkpoint(fn, *args, use_reentrant=False)
    return fn(*args)


class TransformerBlock(nn.Module):
    """Pre-norm block: x + attn(norm1(x)), then + mlp(norm2(x)).

    Parity: nuvla_forge/model/nuvla.py:47-59 (RMSNorm, fused-qkv attention,
    SwiGLU with hidden 4*dim by default). ``grad_checkpoint = True`` recomputes the
    block in backward, on the fused (``forward_chain``) and the unfused path alike.
    """

    def __init__(self, dim: int, heads: int, fused: bool = True, kv_heads: int | None = None,
                 ffn: int | None = None, causal: bool = False):
        super().__init__()
        self.norm1 = RMSNorm(dim, fused=fused)
        self.attn = Attention(dim, heads, kv_heads=kv_heads, causal=causal, fused=fused)
        self.norm2 = RMSNorm(dim, fused=fused)
        self.mlp = SwiGLUMLP(dim, ffn or dim * 4, fused=fused)
        self.grad_checkpoint = False

    def forward(self, x):
        return checkpointed(self, self._forward, x)

    def _forward(self, x):
        x = self.attn(self.norm1(x), residual=x)
        return self.mlp(self.norm2(x), residual=x)

    def forward_chain(self, x, pending=None):
        """Same block with every residual add folded into the following RMSNorm kernel.

        ``pending`` is the previous block's MLP output not yet added to ``x``.
        Returns (x, this block's MLP output, not yet added).
        """
        return checkpointed(self, self._chain, x, pending)

    def _chain(self, x, pending):
        ref = not self.norm1.fused
        if pending is None:
            h = self.norm1(x)
        else:
            x, h = add_rmsnorm(x, pending, self.norm1.weight, self.norm1.eps, force_reference=ref)
        x, h = add_rmsnorm(x, self.attn(h), self.norm2.weight, self.norm2.eps, force_reference=ref)
        return x, self.mlp(h)


def run_blocks(blocks, x, final_norm: RMSNorm | None = None):
    """Run a stack of TransformerBlocks with residual adds fused into the norms.

    Returns final_norm(x_out) when ``final_norm`` is given, else x_out.
    """
    pending = None
    for blk in blocks:
        x, pending = blk.forward_chain(x, pending)
    if pending is None:
        return final_norm(x) if final_norm is not None else x
    if final_norm is None:
        return x + pending
    _, out = add_rmsnorm(x, pending, final_norm.weight, final_norm.eps, force_reference=not final_norm.fused)
    return out

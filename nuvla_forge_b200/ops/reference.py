"""Pure-PyTorch reference implementations (test oracle and CPU fallback).

Every native kernel in :mod:`nuvla_forge_b200.ops` has an fp32-computing
reference here. Parity: nuvla_forge/kernels/reference.py:22-96 (same functions
and signatures for the three fused ops), plus references for the ops the
reference left to PyTorch (attention, RMSNorm, image normalisation, patchify).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def _per_row(c: torch.Tensor, tokens_per_sample: int) -> torch.Tensor:
    """[B, N] per-sample vector -> [B*T, N], row m taking sample m // T."""
    return torch.repeat_interleave(c, tokens_per_sample, dim=0)


def adaln_residual_rmsnorm_ref(x, y, gate, weight, scale, shift, tokens_per_sample: int, eps: float = 1e-6):
    """h = x + gate*y; out = rmsnorm(h) * weight * (1 + scale) + shift.

    x, y: [M, N]; gate, scale, shift: [B, N] with M = B * tokens_per_sample;
    weight: [N]. Returns (h, out) in x's dtype.
    """
    g = _per_row(gate, tokens_per_sample).to(torch.float32)
    s = _per_row(scale, tokens_per_sample).to(torch.float32)
    sh = _per_row(shift, tokens_per_sample).to(torch.float32)
    h = (x.to(torch.float32) + g * y.to(torch.float32)).to(x.dtype)
    hf = h.to(torch.float32)
    inv = torch.rsqrt(hf.square().mean(dim=-1, keepdim=True) + eps)
    out = hf * inv * weight.to(torch.float32) * (1.0 + s) + sh
    return h, out.to(x.dtype)


def rmsnorm_ref(x, weight, eps: float = 1e-6):
    xf = x.to(torch.float32)
    inv = torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + eps)
    return (xf * inv * weight.to(torch.float32)).to(x.dtype)


def add_rmsnorm_ref(x, y, weight, eps: float = 1e-6):
    """h = x + y; out = rmsnorm(h) * weight. Returns (h, out)."""
    h = (x.to(torch.float32) + y.to(torch.float32)).to(x.dtype)
    return h, rmsnorm_ref(h, weight, eps)


def swiglu_ref(a, b):
    """silu(a) * b computed in fp32, returned in a's dtype."""
    return (F.silu(a.to(torch.float32)) * b.to(torch.float32)).to(a.dtype)


def chunked_cross_entropy_ref(hidden, lm_weight, targets, ignore_index: int = -100):
    """Unchunked mean cross entropy over hidden @ lm_weight.T, in fp32."""
    logits = hidden.to(torch.float32) @ lm_weight.to(torch.float32).t()
    return F.cross_entropy(logits, targets, ignore_index=ignore_index, reduction="mean")


def attention_ref(q, k, v, causal: bool = False, scale: float | None = None):
    """Softmax attention in fp32. q [B, Hq, S, D], k/v [B, Hkv, L, D] (GQA when Hkv < Hq)."""
    hq, hkv = q.shape[1], k.shape[1]
    if hkv != hq:
        rep = hq // hkv
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    qf, kf, vf = (t.to(torch.float32) for t in (q, k, v))
    sc = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    s = torch.einsum("bhsd,bhld->bhsl", qf, kf) * sc
    if causal:
        S, L = s.shape[-2], s.shape[-1]
        mask = torch.ones(S, L, dtype=torch.bool, device=s.device).tril(L - S)
        s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhsl,bhld->bhsd", p, vf).to(q.dtype)


def normalise_images_ref(images, dtype=torch.bfloat16, mean=IMAGENET_MEAN, std=IMAGENET_STD):
    """uint8 [..., 3, H, W] -> (v/255 - mean[c]) / std[c] in ``dtype``."""
    x = images.to(torch.float32) / 255.0
    m = torch.tensor(mean, dtype=torch.float32, device=x.device).view(3, 1, 1)
    s = torch.tensor(std, dtype=torch.float32, device=x.device).view(3, 1, 1)
    return ((x - m) / s).to(dtype)


def patchify_ref(images_hwc, patch: int, kpad: int | None = None, dtype=torch.bfloat16,
                 mean=IMAGENET_MEAN, std=IMAGENET_STD):
    """uint8 [n, H, W, 3] -> normalised patch rows [n, (H/p)*(W/p), kpad] in (c, ky, kx) order."""
    n, H, W, _ = images_hwc.shape
    p = patch
    x = images_hwc.to(torch.float32) / 255.0
    m = torch.tensor(mean, dtype=torch.float32, device=x.device)
    s = torch.tensor(std, dtype=torch.float32, device=x.device)
    x = (x - m) / s                                        # [n, H, W, 3]
    x = x.view(n, H // p, p, W // p, p, 3).permute(0, 1, 3, 5, 2, 4)  # [n, hp, wp, 3, p, p]
    x = x.reshape(n, (H // p) * (W // p), 3 * p * p)
    k = 3 * p * p
    if kpad is not None and kpad > k:
        x = F.pad(x, (0, kpad - k))
    return x.to(dtype)

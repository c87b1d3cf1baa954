"""Native flash-attention forward on tcgen05 (csrc/attention.cu).

``attention_fwd(q, k, v, causal, scale)`` runs the sm_100a kernel on the
projection-native [B, S, H, D] layout and returns (out [B, S, Hq, D], lse
[B, Hq, S]) or None when the inputs are outside what it supports (bf16, D in
{64, 128}, 16-byte-aligned rows, Hkv dividing Hq).

``enable()`` (or ``NFB_ATTN_NATIVE=1`` at import) routes ``ops.attention``
through it. Its backward recomputes the forward with PyTorch SDPA and
differentiates that, so training is correct but pays one extra attention
forward; the cuDNN path stays the default for training until the native
backward exists.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from .. import _native as nat
from .attention import register_native

_status: dict[int, torch.Tensor] = {}


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _status:
        _status[idx] = torch.zeros(1, dtype=torch.int32, device=device)
    return _status[idx]


def check_status(device: torch.device | None = None) -> None:
    device = device or torch.device("cuda", torch.cuda.current_device())
    v = int(_status_word(device).item())
    if v:
        raise RuntimeError(f"native attention gave up waiting (status {v:#x})")


def supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    if not (nat.HAS_NATIVE and q.is_cuda and q.dtype == torch.bfloat16 and k.dtype == q.dtype and v.dtype == q.dtype):
        return False
    if q.dim() != 4 or q.shape[-1] not in (64, 128) or k.shape[-1] != q.shape[-1] or v.shape[-1] != q.shape[-1]:
        return False
    if q.shape[2] % k.shape[2] or k.shape[2] != v.shape[2] or k.shape[1] != v.shape[1]:
        return False
    for t in (q, k, v):
        if t.stride(-1) != 1 or t.data_ptr() % 16 or any(s % 8 for s in t.stride()[:3]):
            return False
    return True


def attention_fwd(q, k, v, causal: bool = False, scale: float | None = None):
    """(out, lse) from the native kernel, or None when unsupported."""
    if not supported(q, k, v):
        return None
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    out = torch.empty((B, Sq, Hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=q.device)
    sc = float(scale) if scale is not None else D ** -0.5
    nat.call("nfb_attn_fwd", nat.ptr(q), nat.ptr(k), nat.ptr(v), nat.ptr(out), nat.ptr(lse), B, Sq, Sk, Hq, Hkv, D,
             q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
             v.stride(0), v.stride(1), v.stride(2), out.stride(0), out.stride(1), out.stride(2),
             int(causal), sc, nat.ptr(_status_word(q.device)), nat.stream(q.device))
    return out, lse


class _NativeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        out, _ = attention_fwd(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v)
        ctx.causal, ctx.scale = causal, scale
        return out

    @staticmethod
    def backward(ctx, g):
        q, k, v = ctx.saved_tensors
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            o = F.scaled_dot_product_attention(qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2),
                                               is_causal=ctx.causal, scale=ctx.scale,
                                               enable_gqa=kk.shape[2] != qq.shape[2]).transpose(1, 2)
            dq, dk, dv = torch.autograd.grad(o, (qq, kk, vv), g)
        return dq, dk, dv, None, None


def _native(q, k, v, causal, scale):
    if not supported(q, k, v):
        return None
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return _NativeAttention.apply(q, k, v, causal, scale)
    return attention_fwd(q, k, v, causal, scale)[0]


def enable(flag: bool = True) -> None:
    """Route ops.attention through the native forward (off by default)."""
    register_native(_native if flag else None)


if os.environ.get("NFB_ATTN_NATIVE", "0") == "1":
    enable(True)

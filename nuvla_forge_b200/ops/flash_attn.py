"""Native flash attention on tcgen05: forward (csrc/attention.cu) and backward (csrc/attention_bwd.cu).

``attention_fwd(q, k, v, causal, scale)`` runs the sm_100a forward on the
projection-native [B, S, H, D] layout and returns (out [B, S, Hq, D], lse
[B, Hq, S]); ``attention_bwd`` returns (dq, dk, dv) from the saved inputs, the
output, its gradient and lse. Both return None when the inputs are outside what
the kernels support (bf16, D in {64, 128}, 16-byte-aligned rows, Hkv dividing
Hq, and for a causal mask Sq == Sk: the kernels align the mask to the bottom
right, which only equals PyTorch's top-left ``is_causal`` for square masks).

Routing of ``ops.attention`` (``NFB_ATTN_NATIVE`` at import, or ``enable(mode)``): ``auto``
(default) uses the native kernels only where they measured faster than cuDNN on B200 -- a short
query sequence attending a long context (at most 128 queries, at least 1024 keys: the DiT's
cross-attention into the backbone states, forward + backward 0.236 vs 0.251 ms at config 3;
reports/attention.json) -- and cuDNN SDPA elsewhere (self-attention over the ViT and backbone
tokens, where the native kernels run at 57-69% of cuDNN's speed); ``1`` uses them wherever they
support the shape, ``0`` never.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.nn.functional as F

from .. import _native as nat
from .attention import register_native

_status: dict[int, torch.Tensor] = {}
# NFB_ATTN_NATIVE_BWD=0 keeps the native forward but differentiates through SDPA (for A/B comparisons)
_NATIVE_BWD = os.environ.get("NFB_ATTN_NATIVE_BWD", "1") == "1"


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


def supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> bool:
    if not (nat.HAS_NATIVE and q.is_cuda and q.dtype == torch.bfloat16 and k.dtype == q.dtype and v.dtype == q.dtype):
        return False
    if causal and q.shape[1] != k.shape[1]:
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
    if not supported(q, k, v, causal):
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


def attention_bwd(q, k, v, out, dout, lse, causal: bool = False, scale: float | None = None):
    """(dq, dk, dv) from the native backward (3 launches), or None when unsupported."""
    if not supported(q, k, v, causal) or dout.dtype != q.dtype or dout.stride(-1) != 1 or dout.data_ptr() % 16 \
            or any(s % 8 for s in dout.stride()[:3]):
        return None
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    dq = torch.empty((B, Sq, Hq, D), dtype=q.dtype, device=q.device)
    dk = torch.empty((B, Sk, Hkv, D), dtype=q.dtype, device=q.device)
    dv = torch.empty((B, Sk, Hkv, D), dtype=q.dtype, device=q.device)
    nbytes = int(nat.lib().nfb_attn_bwd_scratch_bytes(B, Sq, Hq, D))
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    st = []
    for t in (q, k, v, out, dout, dq, dk, dv):
        st += [t.stride(0), t.stride(1), t.stride(2)]
    strides = (ctypes.c_int64 * 24)(*st)
    sc = float(scale) if scale is not None else D ** -0.5
    nat.call("nfb_attn_bwd", nat.ptr(q), nat.ptr(k), nat.ptr(v), nat.ptr(out), nat.ptr(dout), nat.ptr(lse),
             nat.ptr(dq), nat.ptr(dk), nat.ptr(dv), nat.ptr(scratch), B, Sq, Sk, Hq, Hkv, D, strides, int(causal), sc,
             nat.ptr(_status_word(q.device)), nat.stream(q.device))
    return dq, dk, dv


class _NativeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        out, lse = attention_fwd(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale = causal, scale
        return out

    @staticmethod
    def backward(ctx, g):
        q, k, v, out, lse = ctx.saved_tensors
        if _NATIVE_BWD:
            res = attention_bwd(q, k, v, out, g.contiguous() if g.stride(-1) != 1 else g, lse, ctx.causal, ctx.scale)
            if res is not None:
                return res[0], res[1], res[2], None, None
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            o = F.scaled_dot_product_attention(qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2),
                                               is_causal=ctx.causal, scale=ctx.scale,
                                               enable_gqa=kk.shape[2] != qq.shape[2]).transpose(1, 2)
            dq, dk, dv = torch.autograd.grad(o, (qq, kk, vv), g)
        return dq, dk, dv, None, None


_MODE = "auto"


def _faster_than_sdpa(q, k) -> bool:
    """The measured regime where the native kernels beat cuDNN: few queries, a long context."""
    return q.shape[1] <= 128 and k.shape[1] >= 1024


def _native(q, k, v, causal, scale):
    if not supported(q, k, v, causal):
        return None
    if _MODE == "auto" and not _faster_than_sdpa(q, k):
        return None
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return _NativeAttention.apply(q, k, v, causal, scale)
    return attention_fwd(q, k, v, causal, scale)[0]


def enable(flag: bool | str = True) -> None:
    """Route ops.attention through the native kernels: True / "1" wherever supported, "auto" where
    they measured faster than cuDNN, False / "0" never."""
    global _MODE
    mode = {True: "1", False: "0"}.get(flag, str(flag))
    if mode not in ("0", "1", "auto"):
        raise ValueError(f"attention routing mode {flag!r}: expected 0, 1 or auto")
    _MODE = mode
    register_native(_native if mode != "0" else None)


enable(os.environ.get("NFB_ATTN_NATIVE", "auto"))

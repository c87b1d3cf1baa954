"""Fused SwiGLU (native kernels in csrc/swiglu.cu).

Parity: nuvla_forge/kernels/swiglu.py:95-106 — ``fused_swiglu(a, b,
force_reference=False)`` for any shape. Added: ``swiglu_packed(ab)`` which
takes the [.., 2F] output of ONE fused gate/up projection (gate columns first)
and whose backward writes d(ab) as one [.., 2F] buffer, so the MLP needs one
input-gradient GEMM instead of two plus an add.
"""

from __future__ import annotations

import torch

from .. import _native as nat
from .reference import swiglu_ref


def _native_ok(t: torch.Tensor) -> bool:
    return nat.HAS_NATIVE and t.is_cuda and t.dtype in (torch.bfloat16, torch.float16, torch.float32)


def _aligned_rows(t: torch.Tensor) -> bool:
    es = t.element_size()
    return t.stride(-1) == 1 and (t.stride(0) * es) % 16 == 0 and t.data_ptr() % 16 == 0


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        shape = a.shape
        n = shape[-1]
        a2 = a.reshape(-1, n).contiguous()
        b2 = b.reshape(-1, n).contiguous()
        m = a2.shape[0]
        out = torch.empty((m, n), dtype=a.dtype, device=a.device)
        nat.call("nfb_swiglu_fwd", nat.dtype_code(a.dtype), nat.ptr(a2), nat.ptr(b2), nat.ptr(out),
                 m, n, n, n, n, nat.stream(a.device))
        ctx.save_for_backward(a2, b2)
        ctx.shape = shape
        return out.view(shape)

    @staticmethod
    def backward(ctx, dout):
        a2, b2 = ctx.saved_tensors
        m, n = a2.shape
        d2 = dout.reshape(m, n).contiguous()
        da = torch.empty_like(a2)
        db = torch.empty_like(b2)
        nat.call("nfb_swiglu_bwd", nat.dtype_code(a2.dtype), nat.ptr(d2), nat.ptr(a2), nat.ptr(b2),
                 nat.ptr(da), nat.ptr(db), m, n, n, n, n, n, n, nat.stream(a2.device))
        return da.view(ctx.shape), db.view(ctx.shape)


class _SwiGLUPacked(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ab):
        two_f = ab.shape[-1]
        f = two_f // 2
        ab2 = ab.reshape(-1, two_f)
        if not _aligned_rows(ab2):
            ab2 = ab2.contiguous()
        m = ab2.shape[0]
        out = torch.empty((m, f), dtype=ab.dtype, device=ab.device)
        a_view, b_view = ab2[:, :f], ab2[:, f:]
        nat.call("nfb_swiglu_fwd", nat.dtype_code(ab.dtype), nat.ptr(a_view), nat.ptr(b_view), nat.ptr(out),
                 m, f, ab2.stride(0), ab2.stride(0), f, nat.stream(ab.device))
        ctx.save_for_backward(ab2)
        ctx.shape = ab.shape
        return out.view(*ab.shape[:-1], f)

    @staticmethod
    def backward(ctx, dout):
        (ab2,) = ctx.saved_tensors
        m, two_f = ab2.shape
        f = two_f // 2
        d2 = dout.reshape(m, f)
        if not _aligned_rows(d2):
            d2 = d2.contiguous()
        dab = torch.empty((m, two_f), dtype=ab2.dtype, device=ab2.device)
        nat.call("nfb_swiglu_bwd", nat.dtype_code(ab2.dtype), nat.ptr(d2), nat.ptr(ab2[:, :f]), nat.ptr(ab2[:, f:]),
                 nat.ptr(dab[:, :f]), nat.ptr(dab[:, f:]), m, f, d2.stride(0), two_f, two_f, two_f, two_f,
                 nat.stream(ab2.device))
        return dab.view(ctx.shape)


def fused_swiglu(a: torch.Tensor, b: torch.Tensor, force_reference: bool = False) -> torch.Tensor:
    """silu(a) * b in one pass (forward and backward)."""
    if force_reference or not _native_ok(a) or a.numel() == 0:
        return swiglu_ref(a, b)
    if b.dtype != a.dtype:
        b = b.to(a.dtype)
    return _SwiGLU.apply(a, b)


def swiglu_packed(ab: torch.Tensor, force_reference: bool = False) -> torch.Tensor:
    """silu(ab[..., :F]) * ab[..., F:] for a packed [.., 2F] gate/up projection output."""
    f = ab.shape[-1] // 2
    if force_reference or not _native_ok(ab) or f % 8 or ab.numel() == 0:
        return swiglu_ref(ab[..., :f], ab[..., f:])
    return _SwiGLUPacked.apply(ab)

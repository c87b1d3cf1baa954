"""Fused residual / RMSNorm / adaLN-Zero ops (native sm_100a kernels, csrc/norm.cu).

One kernel family covers every normalisation seam of the model:

* ``rmsnorm(x, w)``                                   out = rmsnorm(x) * w
* ``rmsnorm(x, w, scale=s, shift=sh, T)``             out = rmsnorm(x) * w * (1 + s[b]) + sh[b]
* ``add_rmsnorm(x, y, w)``                            h = x + y;        out = rmsnorm(h) * w
* ``fused_adaln_residual_rmsnorm(x, y, g, w, s, sh, T)``  h = x + g[b]*y; out = rmsnorm(h)*w*(1+s[b])+sh[b]

Parity: nuvla_forge/kernels/adaln_rmsnorm.py:239-270 (same public signature,
same (h, out) return, same ``force_reference`` escape hatch). ``gate=None``
means a gate of one and ``scale=shift=None`` means no modulation, which the
reference expressed with zero/one buffers (nuvla_forge/model/dit.py:141-142).

Backward is one deterministic launch (see csrc/norm.cu). Per-sample
conditioning tensors may be strided row views (for example ``cond(c).chunk(6)``
outputs) and are read in place, without ``.contiguous()`` copies.
"""

from __future__ import annotations

import torch

from .. import _native as nat
from .reference import adaln_residual_rmsnorm_ref, rmsnorm_ref

GATE_NONE, GATE_ONE, GATE_VEC = 0, 1, 2
MAX_N = 8192

_tickets: dict[int, torch.Tensor] = {}
_status: dict[int, torch.Tensor] = {}
_impl_set = [False]


class NormTimeout(RuntimeError):
    """A pipelined norm kernel gave up waiting for its row copies (bounded wait expired)."""


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def _ensure_native_state(device: torch.device) -> None:
    """Register this device's status word with the kernels and apply ``NFB_NORM_IMPL`` once.

    The default (``NFB_NORM_IMPL=0``) is the register-resident warp/team
    kernels; ``1`` selects the bulk-copy pipelined kernels where rows allow
    (slower on B200 at the model's shapes; kept for comparison).
    """
    idx = _dev_index(device)
    if idx not in _status:
        _status[idx] = torch.zeros(1, dtype=torch.int32, device=device)
        with torch.cuda.device(idx):
            nat.lib().nfb_norm_set_status(nat.ptr(_status[idx]))
    if not _impl_set[0]:
        import os
        set_impl(int(os.environ.get("NFB_NORM_IMPL", "0")))


def set_impl(impl: int) -> None:
    """Select the norm kernel family: 0 = warp/team (default), 1 = bulk-copy pipelined."""
    nat.lib().nfb_norm_set_impl(int(impl))
    _impl_set[0] = True
    _bwd_ctas.clear()


def get_impl() -> int:
    return int(nat.lib().nfb_norm_get_impl())


_bwd_ctas: dict[tuple[int, int, int], int] = {}


def _bwd_P(M: int, N: int, B: int) -> int:
    """CTAs per sample of the backward (depends on the shape, the SM count and the kernel family)."""
    key = (M, N, B)
    P = _bwd_ctas.get(key)
    if P is None:
        P = _bwd_ctas[key] = int(nat.lib().nfb_norm_bwd_P(M, N, B))
    return P


def check_status(device: torch.device | None = None) -> None:
    """Raise :class:`NormTimeout` if a pipelined norm kernel on ``device`` timed out (synchronises)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    st = _status.get(_dev_index(device))
    if st is not None and int(st.item()) != 0:
        v = int(st.item())
        st.zero_()
        raise NormTimeout(f"norm kernel copy wait timed out (status 0x{v:08x}, site {v & 0xFFFFFF})")


def ticket_buffer(device: torch.device, n: int) -> torch.Tensor:
    """Zeroed uint32 ticket counters the kernels leave zeroed (persistent per device)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _tickets.get(idx)
    if buf is None or buf.numel() < n:
        buf = torch.zeros(max(n, 4096), dtype=torch.int32, device=device)
        _tickets[idx] = buf
    return buf


def _rows(t: torch.Tensor, n: int) -> torch.Tensor:
    """2-D [rows, n] view with unit column stride and a 16-byte-aligned row stride."""
    if t.dim() != 2:
        t = t.reshape(-1, n)
    if t.is_contiguous():  # rows of n % 8 == 0 elements keep every row 16-byte aligned
        return t if t.data_ptr() % 16 == 0 else t.clone()
    es = t.element_size()
    if t.stride(1) != 1 or (t.stride(0) * es) % 16 or t.data_ptr() % 16:
        t = t.contiguous()  # t is not contiguous here, so this copies into a fresh (aligned) allocation
    return t


def _native_ok(x: torch.Tensor) -> bool:
    n = x.shape[-1]
    return (nat.HAS_NATIVE and x.is_cuda and x.dtype in (torch.bfloat16, torch.float16, torch.float32)
            and n % 8 == 0 and n <= MAX_N)


def _wflag(weight: torch.Tensor, x: torch.Tensor) -> tuple[torch.Tensor, int]:
    if weight.dtype == torch.float32:
        return weight.contiguous(), 1
    if weight.dtype != x.dtype:
        weight = weight.to(x.dtype)
    return weight.contiguous(), 0


def _fwd(x, y, gate, weight, scale, shift, T, eps, gate_mode, mod):
    M, N = x.shape
    _ensure_native_state(x.device)
    w, wf = _wflag(weight, x)
    h = torch.empty((M, N), dtype=x.dtype, device=x.device) if gate_mode != GATE_NONE else None
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    rstd = torch.empty(M, dtype=torch.float32, device=x.device)
    nat.call(
        "nfb_norm_fwd", nat.dtype_code(x.dtype), gate_mode, int(mod),
        nat.ptr(x), nat.ptr(y), nat.ptr(gate), nat.ptr(w), nat.ptr(scale), nat.ptr(shift),
        nat.ptr(h), nat.ptr(out), nat.ptr(rstd),
        M, N, T,
        x.stride(0), y.stride(0) if y is not None else 0, N, N,
        gate.stride(0) if gate is not None else 0,
        scale.stride(0) if scale is not None else 0,
        shift.stride(0) if shift is not None else 0,
        float(eps), wf, nat.stream(x.device),
    )
    return h, out, rstd, w, wf


def _bwd(ctx, dh_up, dout):
    hs, y, gate, w, scale, rstd = ctx.saved_tensors
    gate_mode, mod, T, wf = ctx.gate_mode, ctx.mod, ctx.T, ctx.wf
    M, N = hs.shape
    B = M // T
    dev = hs.device
    _ensure_native_state(dev)
    if dout is None:
        dout = torch.zeros_like(hs)
    dout = _rows(dout, N)
    if dh_up is not None:
        dh_up = _rows(dh_up, N)
    P = _bwd_P(M, N, B)
    partials = torch.empty(B * P * 3 * N, dtype=torch.float32, device=dev)
    dwb = torch.empty(B * N, dtype=torch.float32, device=dev)
    tickets = ticket_buffer(dev, B + 1)
    dx = torch.empty((M, N), dtype=hs.dtype, device=dev)
    # with a gate of one, dy == dx: the kernel writes it once and both inputs share the tensor
    dy = torch.empty((M, N), dtype=hs.dtype, device=dev) if gate_mode == GATE_VEC else None
    dgate = torch.empty((B, N), dtype=hs.dtype, device=dev) if gate_mode == GATE_VEC else None
    dscale = torch.empty((B, N), dtype=hs.dtype, device=dev) if mod else None
    dshift = torch.empty((B, N), dtype=hs.dtype, device=dev) if mod else None
    dweight = torch.empty(N, dtype=w.dtype, device=dev)
    nat.call(
        "nfb_norm_bwd", nat.dtype_code(hs.dtype), gate_mode, int(mod),
        nat.ptr(dh_up), nat.ptr(dout), nat.ptr(hs), nat.ptr(y), nat.ptr(gate), nat.ptr(w), nat.ptr(scale),
        nat.ptr(rstd), nat.ptr(dx), nat.ptr(dy), nat.ptr(dgate), nat.ptr(dscale), nat.ptr(dshift),
        nat.ptr(dweight), nat.ptr(partials), nat.ptr(dwb), nat.ptr(tickets),
        M, N, T, P,
        dh_up.stride(0) if dh_up is not None else 0, dout.stride(0), hs.stride(0),
        y.stride(0) if y is not None else 0, N, N,
        gate.stride(0) if gate is not None else 0, scale.stride(0) if scale is not None else 0,
        wf, nat.stream(dev),
    )
    return dx, dy, dgate, dweight, dscale, dshift


class _NormFn(torch.autograd.Function):
    """out = rmsnorm(x) * w [* (1 + scale[b]) + shift[b]]"""

    @staticmethod
    def forward(ctx, x, weight, scale, shift, T, eps):
        mod = scale is not None
        _, out, rstd, w, wf = _fwd(x, None, None, weight, scale, shift, T, eps, GATE_NONE, mod)
        ctx.save_for_backward(x, None, None, w, scale, rstd)
        ctx.gate_mode, ctx.mod, ctx.T, ctx.wf = GATE_NONE, mod, T, wf
        ctx.wdtype = weight.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        dx, _, _, dweight, dscale, dshift = _bwd(ctx, None, dout)
        return dx, dweight.to(ctx.wdtype), dscale, dshift, None, None


class _ResNormFn(torch.autograd.Function):
    """h = x + g*y; out = rmsnorm(h) * w [* (1 + scale[b]) + shift[b]]"""

    @staticmethod
    def forward(ctx, x, y, gate, weight, scale, shift, T, eps):
        gate_mode = GATE_VEC if gate is not None else GATE_ONE
        mod = scale is not None
        h, out, rstd, w, wf = _fwd(x, y, gate, weight, scale, shift, T, eps, gate_mode, mod)
        ctx.save_for_backward(h, y if gate_mode == GATE_VEC else None, gate, w, scale, rstd)
        ctx.gate_mode, ctx.mod, ctx.T, ctx.wf = gate_mode, mod, T, wf
        ctx.wdtype = weight.dtype
        return h, out

    @staticmethod
    def backward(ctx, dh, dout):
        dx, dy, dgate, dweight, dscale, dshift = _bwd(ctx, dh, dout)
        if ctx.gate_mode == GATE_ONE:
            dy = dx
        return dx, dy, dgate, dweight.to(ctx.wdtype), dscale, dshift, None, None


def _cond(c, n, dtype):
    if c is None:
        return None
    if c.dtype != dtype:
        c = c.to(dtype)
    return _rows(c, n)


def rmsnorm(x, weight, eps: float = 1e-6, scale=None, shift=None, tokens_per_sample: int | None = None,
            force_reference: bool = False):
    """RMSNorm over the last dim, optionally followed by adaLN modulation with [B, N] scale/shift."""
    n = x.shape[-1]
    shape = x.shape
    if (scale is None) != (shift is None):
        raise ValueError("scale and shift must be given together")
    if force_reference or not _native_ok(x):
        out = rmsnorm_ref(x, weight, eps)
        if scale is not None:
            T = tokens_per_sample or (x.reshape(-1, n).shape[0] // scale.shape[0])
            s = torch.repeat_interleave(scale, T, dim=0).view(shape)
            sh = torch.repeat_interleave(shift, T, dim=0).view(shape)
            out = (out.float() * (1 + s.float()) + sh.float()).to(x.dtype)
        return out
    x2 = _rows(x, n)
    M = x2.shape[0]
    if scale is not None:
        T = tokens_per_sample or (M // scale.shape[0])
    else:
        T = M if M > 0 else 1
    out = _NormFn.apply(x2, weight, _cond(scale, n, x.dtype), _cond(shift, n, x.dtype), T, eps)
    return out.view(shape)


def add_rmsnorm(x, y, weight, eps: float = 1e-6, force_reference: bool = False):
    """h = x + y; out = rmsnorm(h) * weight. Returns (h, out)."""
    n = x.shape[-1]
    shape = x.shape
    if force_reference or not _native_ok(x):
        h = (x.float() + y.float()).to(x.dtype)
        return h, rmsnorm_ref(h, weight, eps)
    x2, y2 = _rows(x, n), _rows(y.to(x.dtype), n)
    M = x2.shape[0]
    h, out = _ResNormFn.apply(x2, y2, None, weight, None, None, M if M > 0 else 1, eps)
    return h.view(shape), out.view(shape)


def fused_adaln_residual_rmsnorm(x, y, gate, weight, scale, shift, tokens_per_sample: int, eps: float = 1e-6,
                                 force_reference: bool = False):
    """Fused gated residual + RMSNorm + adaLN-Zero modulation.

    x, y: [M, N] (or [B, T, N]); gate, scale, shift: [B, N] or None; weight: [N].
    Returns (h, out) with h = x + gate*y and out = rmsnorm(h)*weight*(1+scale)+shift.
    """
    n = x.shape[-1]
    shape = x.shape
    if (scale is None) != (shift is None):
        raise ValueError("scale and shift must be given together")
    if force_reference or not _native_ok(x):
        B = x.reshape(-1, n).shape[0] // tokens_per_sample
        g = gate if gate is not None else torch.ones(B, n, dtype=x.dtype, device=x.device)
        s = scale if scale is not None else torch.zeros(B, n, dtype=x.dtype, device=x.device)
        sh = shift if shift is not None else torch.zeros(B, n, dtype=x.dtype, device=x.device)
        h, out = adaln_residual_rmsnorm_ref(x.reshape(-1, n), y.reshape(-1, n), g, weight, s, sh,
                                            tokens_per_sample, eps)
        return h.view(shape), out.view(shape)
    x2, y2 = _rows(x, n), _rows(y.to(x.dtype), n)
    h, out = _ResNormFn.apply(x2, y2, _cond(gate, n, x.dtype), weight, _cond(scale, n, x.dtype),
                              _cond(shift, n, x.dtype), tokens_per_sample, eps)
    return h.view(shape), out.view(shape)

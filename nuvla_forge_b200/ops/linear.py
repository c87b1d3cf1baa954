"""Linear layers on the CTA-pair tcgen05 GEMM (native csrc/gemm.cu).

Parity: the reference's linear layers are ``nn.Linear`` / ``F.linear`` on cuBLAS
(nuvla_forge/model/dit.py:75-76, 91-92, 99-101, nuvla_forge/model/nuvla.py:112, 123).
Here all three GEMMs of a linear layer run on one native kernel family:

* forward ``y = x W^T (+ b) (+ residual)``: bias and residual are added in the
  epilogue (the residual replaces cuBLAS's ``addmm`` C operand);
* input gradient ``dx = dy W``: W read MN-major, no transposed copy;
* weight gradient ``dW = dy^T x``: both operands MN-major, fp32 accumulation,
  split over the token dimension with the slices added in a fixed order (the
  result is bit-identical from run to run).

When the weight's owner (the DDP / FSDP runtime) registered a gradient sink on
the parameter, the weight gradient is written (or added) straight into the
owner's fp32 gradient buffer and the owner is told the gradient is complete:
no bf16 gradient tensor and no separate accumulation kernel exist. Without an
owner, the fp32 result is cast to the parameter dtype and returned to autograd.

Layers whose widths the tensor-core kernel cannot tile (the 3-wide waypoint
projections of the DiT) run all three products on a small CUDA-core kernel of
the same library. CPU tensors run ``F.linear``; so does everything when
``NFB_LINEAR=cublas`` is set, for A/B comparisons.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from .. import _native as nat

_status: dict[int, torch.Tensor] = {}
_flags: dict[int, torch.Tensor] = {}
_epoch = [0]

FLAG_WORDS = 1 << 16      # split-K flags: 8 per 256 x 256 tile, any weight up to 8192 tiles


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def status_word(device: torch.device) -> torch.Tensor:
    idx = _dev_index(device)
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _status[idx] = t
    return t


def check_status(device: torch.device | None = None) -> None:
    """Raise if a GEMM's bounded pipeline wait gave up on any device since the start."""
    for idx, t in _status.items():
        v = int(t.item())
        if v:
            raise RuntimeError(f"tcgen05 GEMM on cuda:{idx} gave up waiting (status {v:#x}, site {v & 0xFFFFFF})")


def _flag_buffer(device: torch.device) -> torch.Tensor:
    idx = _dev_index(device)
    t = _flags.get(idx)
    if t is None:
        t = torch.zeros(FLAG_WORDS, dtype=torch.int32, device=device)
        _flags[idx] = t
    return t


def native_enabled() -> bool:
    return nat.HAS_NATIVE and os.environ.get("NFB_LINEAR", "native") != "cublas"


def _rows_ok(t: torch.Tensor) -> bool:
    """2-D, unit inner stride, 16-byte aligned base and rows."""
    return (t.dim() == 2 and t.stride(1) == 1 and t.data_ptr() % 16 == 0 and (t.stride(0) * t.element_size()) % 16 == 0
            and t.shape[1] % 8 == 0)


def _aligned_rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` itself when the TMA can read it in place, else a packed, 16-byte aligned copy."""
    if _rows_ok(t):
        return t
    t = t.contiguous()
    return t if _rows_ok(t) else t.clone()


def _describe(t: torch.Tensor | None) -> str:
    if t is None:
        return "None"
    return f"{tuple(t.shape)} strides {t.stride()} {t.dtype} ptr%16={t.data_ptr() % 16}"


def supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (native_enabled() and x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
            and w.dim() == 2 and w.stride(1) == 1 and w.shape[0] % 8 == 0 and w.shape[1] % 8 == 0
            and w.data_ptr() % 16 == 0 and (w.stride(0) * 2) % 16 == 0)


# ----------------------------------------------------------------------------- raw GEMMs
def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False,
         out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
         bias: torch.Tensor | None = None, residual: torch.Tensor | None = None) -> torch.Tensor:
    """C = A B^T (+ bias) (+ residual) on the CTA-pair tcgen05 kernel.

    ``a`` is A [M, K] (K contiguous) or, with ``a_mn``, A stored as [K, M]; ``b`` is
    B [N, K] or, with ``b_mn``, B stored as [K, N]. bf16 operands; C bf16 or fp32.
    """
    M, K = (a.shape[1], a.shape[0]) if a_mn else (a.shape[0], a.shape[1])
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    ldr = residual.stride(0) if residual is not None else 0
    try:
        nat.call("nfb_gemm", nat.ptr(a), nat.ptr(b), nat.ptr(out), M, N, K, a.stride(0), b.stride(0),
                 out.stride(0), int(a_mn), int(b_mn), int(out.dtype == torch.float32), nat.ptr(bias),
                 nat.ptr(residual), ldr, nat.ptr(status_word(a.device)), nat.stream(a.device))
    except nat.NativeError as e:
        raise nat.NativeError(f"{e}; A {_describe(a)} a_mn={a_mn}, B {_describe(b)} b_mn={b_mn}, "
                              f"C {_describe(out)}, residual {_describe(residual)}") from None
    return out


def gemm_acc(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False,
             accumulate: bool = False, splits: int = 0) -> torch.Tensor:
    """fp32 ``c`` = A B^T (or += with ``accumulate``), split over K in a fixed summation order."""
    M, K = (a.shape[1], a.shape[0]) if a_mn else (a.shape[0], a.shape[1])
    N = b.shape[1] if b_mn else b.shape[0]
    flags = _flag_buffer(a.device)
    _epoch[0] = (_epoch[0] + 1) & 0xFFFFFF
    nat.call("nfb_gemm_acc", nat.ptr(a), nat.ptr(b), nat.ptr(c), M, N, K, a.stride(0), b.stride(0), c.stride(0),
             int(a_mn), int(b_mn), int(accumulate), int(splits), nat.ptr(flags), flags.numel(), _epoch[0],
             nat.ptr(status_word(a.device)), nat.stream(a.device))
    return c


# ----------------------------------------------------------------------------- autograd
def weight_grad(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor):
    """dW = dy^T x for weight ``w``; into the owner's fp32 buffer when one is registered.

    An owner is any object set as ``w._nfb_grad_owner`` with ``grad_target(w) ->
    (fp32 buffer of w's numel, overwrite)`` and ``grad_done(w)``. Returns the
    gradient to hand to autograd (None when the owner received it).
    """
    owner = getattr(w, "_nfb_grad_owner", None)
    if owner is not None:
        buf, overwrite = owner.grad_target(w)
        gemm_acc(dy2, x2, buf.view(w.shape[0], w.shape[1]), a_mn=True, b_mn=True, accumulate=not overwrite)
        owner.grad_done(w)
        return None
    g = torch.empty(w.shape, dtype=torch.float32, device=w.device)
    gemm_acc(dy2, x2, g, a_mn=True, b_mn=True, accumulate=False)
    return g.to(w.dtype)


def input_grad(dy2: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """dx = dy W (W [N, K] read as an MN-major operand)."""
    return gemm(dy2, w, b_mn=True)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, bias, residual):
        K = x.shape[-1]
        x2 = _aligned_rows(x.reshape(-1, K))
        r2 = None
        if residual is not None:
            r2 = _aligned_rows(residual.reshape(-1, w.shape[0]))
        y = gemm(x2, w, bias=bias, residual=r2)
        ctx.save_for_backward(x2, w)
        ctx.w_ref = w          # the Parameter object itself (its gradient owner is an attribute)
        ctx.x_shape = x.shape
        ctx.has_bias = bias is not None
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = _aligned_rows(dy.reshape(-1, w.shape[0]))
        dx = dw = db = dr = None
        if ctx.needs_input_grad[0]:
            dx = input_grad(dy2, w).view(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            dw = weight_grad(dy2, x2, ctx.w_ref)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = dy2.float().sum(0).to(dy.dtype)
        if ctx.has_res and ctx.needs_input_grad[3]:
            dr = dy
        return dx, dw, db, dr


# ----------------------------------------------------------------------------- SwiGLU MLP
def interleave_gate_up(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """[gate; up] rows -> 128-row blocks (gate block b, up block b, ...), the fused kernel's layout."""
    F, D = g.shape
    return torch.stack([g.reshape(F // 128, 128, D), u.reshape(F // 128, 128, D)], dim=1).reshape(2 * F, D)


def split_gate_up_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of :func:`interleave_gate_up`: (gate rows, up rows) of an interleaved weight."""
    F2, D = w.shape
    v = w.reshape(F2 // 256, 2, 128, D)
    return v[:, 0].reshape(F2 // 2, D), v[:, 1].reshape(F2 // 2, D)


def split_gate_up_cols(ab: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(gate, up) columns of a pre-activation computed with an interleaved weight (copies)."""
    F2 = ab.shape[-1]
    v = ab.reshape(*ab.shape[:-1], F2 // 256, 2, 128)
    return v[..., 0, :].reshape(*ab.shape[:-1], F2 // 2), v[..., 1, :].reshape(*ab.shape[:-1], F2 // 2)


def swiglu_supported(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor) -> bool:
    return (supported(x, w_gu) and supported(x, w_down) and w_gu.shape[0] % 256 == 0 and x.numel() > 0
            and w_down.shape[1] * 2 == w_gu.shape[0] and w_gu.is_contiguous() and w_down.is_contiguous())


class _SwiGluMLPFn(torch.autograd.Function):
    """y = W_down (silu(gate) * up) (+ residual), gate/up = x W_gu^T, W_gu interleaved in 128-row blocks.

    Forward: one GEMM whose epilogue writes the pre-activations and the activation, then the down
    projection (residual in its epilogue). Backward: the down projection's input gradient with the
    SwiGLU backward in its epilogue (d_act never stored), then the weight gradients and the input
    gradient of the gate/up projection.
    """

    @staticmethod
    def forward(ctx, x, w_gu, w_down, residual):
        K = x.shape[-1]
        F2 = w_gu.shape[0]
        F = F2 // 2
        D = w_down.shape[0]
        x2 = _aligned_rows(x.reshape(-1, K))
        M = x2.shape[0]
        ab = torch.empty((M, F2), dtype=x.dtype, device=x.device)
        act = torch.empty((M, F), dtype=x.dtype, device=x.device)
        st = status_word(x.device)
        nat.call("nfb_gemm_swiglu_fwd", nat.ptr(x2), nat.ptr(w_gu), nat.ptr(ab), nat.ptr(act), M, F, K, x2.stride(0),
                 w_gu.stride(0), ab.stride(0), act.stride(0), nat.ptr(st), nat.stream(x.device))
        r2 = _aligned_rows(residual.reshape(-1, D)) if residual is not None else None
        y = gemm(act, w_down, residual=r2)
        ctx.save_for_backward(x2, w_gu, w_down, ab, act)
        ctx.w_refs = (w_gu, w_down)
        ctx.x_shape = x.shape
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], D)

    @staticmethod
    def backward(ctx, dy):
        x2, w_gu, w_down, ab, act = ctx.saved_tensors
        w_gu_ref, w_down_ref = ctx.w_refs
        M, F2 = ab.shape
        F = F2 // 2
        D = w_down.shape[0]
        dy2 = _aligned_rows(dy.reshape(-1, D))
        dab = torch.empty_like(ab)
        nat.call("nfb_gemm_swiglu_bwd", nat.ptr(dy2), nat.ptr(w_down), nat.ptr(ab), nat.ptr(dab), M, F, D,
                 dy2.stride(0), w_down.stride(0), ab.stride(0), dab.stride(0), nat.ptr(status_word(dy.device)),
                 nat.stream(dy.device))
        dx = dw_gu = dw_down = dr = None
        if ctx.needs_input_grad[2]:
            dw_down = weight_grad(dy2, act, w_down_ref)
        if ctx.needs_input_grad[0]:
            dx = input_grad(dab, w_gu).view(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            dw_gu = weight_grad(dab, x2, w_gu_ref)
        if ctx.has_res and ctx.needs_input_grad[3]:
            dr = dy
        return dx, dw_gu, dw_down, dr


def swiglu_mlp(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor,
               residual: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU MLP with the activation fused into the GEMM epilogues (see :class:`_SwiGluMLPFn`)."""
    return _SwiGluMLPFn.apply(x, w_gu, w_down, residual)


def gemm_small(a: torch.Tensor, sa: tuple, b: torch.Tensor, sb: tuple, c: torch.Tensor, sc: tuple,
               M: int, N: int, K: int, bias: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """C[m, n] (+)= sum_k A[m, k] B[n, k] (+ bias) on CUDA cores; s* = (row, column) element strides."""
    nat.call("nfb_gemm_small", nat.dtype_code(a.dtype), int(c.dtype == torch.float32), nat.ptr(a), sa[0], sa[1],
             nat.ptr(b), sb[0], sb[1], nat.ptr(c), sc[0], sc[1], nat.ptr(bias), M, N, K, int(accumulate),
             nat.stream(a.device))
    return c


class _SmallLinearFn(torch.autograd.Function):
    """Linear layer of a width the tensor-core tiles cannot cover (CUDA-core kernel, fp32 sums)."""

    @staticmethod
    def forward(ctx, x, w, bias):
        K = x.shape[-1]
        N = w.shape[0]
        x2 = x.reshape(-1, K).contiguous()
        wc = w.contiguous()
        M = x2.shape[0]
        y = torch.empty((M, N), dtype=x.dtype, device=x.device)
        gemm_small(x2, (K, 1), wc, (K, 1), y, (N, 1), M, N, K, bias=bias)
        ctx.save_for_backward(x2, wc)
        ctx.x_shape = x.shape
        ctx.has_bias = bias is not None
        ctx.w_ref = w
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        M, K = x2.shape
        N = w.shape[0]
        dy2 = dy.reshape(-1, N).contiguous()
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty((M, K), dtype=dy.dtype, device=dy.device)
            gemm_small(dy2, (N, 1), w, (1, K), dx, (K, 1), M, K, N)
            dx = dx.view(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            owner = getattr(ctx.w_ref, "_nfb_grad_owner", None)
            if owner is not None:
                buf, overwrite = owner.grad_target(ctx.w_ref)
                gemm_small(dy2, (1, N), x2, (1, K), buf, (K, 1), N, K, M, accumulate=not overwrite)
                owner.grad_done(ctx.w_ref)
            else:
                g = torch.empty((N, K), dtype=torch.float32, device=dy.device)
                gemm_small(dy2, (1, N), x2, (1, K), g, (K, 1), N, K, M)
                dw = g.to(w.dtype)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = dy2.float().sum(0).to(dy.dtype)
        return dx, dw, db


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
           residual: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T (+ b) (+ residual)`` with all three GEMMs on the native kernels when on a GPU."""
    if x.numel() > 0 and supported(x, w) and (b is None or (b.dtype == torch.bfloat16 and b.is_contiguous())) \
            and (residual is None or residual.dtype == torch.bfloat16):
        return _LinearFn.apply(x, w, b, residual)
    if (native_enabled() and x.is_cuda and x.numel() > 0 and x.dtype == w.dtype and x.dtype in (torch.bfloat16, torch.float32)
            and w.dim() == 2 and (b is None or (b.dtype == x.dtype and b.is_contiguous()))
            and (x.shape[-1] < 64 or w.shape[0] < 64)):
        y = _SmallLinearFn.apply(x, w, b)
        return y if residual is None else y + residual
    y = F.linear(x, w, b)
    return y if residual is None else y + residual

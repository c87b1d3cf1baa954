"""Cross entropy on the tcgen05 GEMM (native csrc/ce_tc.cu).

The [M, V] logits live only in tensor memory: pass 1 turns each 128x256 logit
tile into per-row online-softmax partials, a merge kernel produces the
log-sum-exp and the per-row losses, and pass 2 recomputes the tile and writes
``(softmax - onehot) / count`` in bf16 for one row chunk at a time, which the
two gradient GEMMs consume on the CTA-pair tcgen05 core of the linear layers
(d_hidden = dl @ W with W read MN-major; d_W += dl^T @ h with both operands
MN-major, accumulated in fp32; ``NFB_CE_TC_GRAD_GEMM=0`` hands them to cuBLAS
instead). Like the reference
(nuvla_forge/kernels/chunked_ce.py:120-182) the gradients are produced during
forward and backward only scales them; unlike it, no fp32 logit tile exists and
nothing synchronises the host.
"""

from __future__ import annotations

import os

import torch

from .. import _native as nat
from . import linear as _linear
from .chunked_ce import count_valid, register_tc

_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _status[idx] = t
    return t


def check_status(device: torch.device | None = None) -> None:
    for idx, t in _status.items():
        v = int(t.item())
        if v:
            raise RuntimeError(f"tcgen05 pipeline on cuda:{idx} gave up waiting (status {v:#x})")


def tc_gemm(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16, a_mn: bool = False, b_mn: bool = False,
            out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """C = A @ B.T on the native tcgen05 core (bf16 operands, fp32 accumulation).

    ``a`` is A [M, K] (K contiguous), or with ``a_mn`` A stored transposed as [K, M];
    ``b`` is B [N, K], or with ``b_mn`` B stored as [K, N]. Rows must be 16-byte aligned
    (contiguous dimension a multiple of 8). ``out`` (optional, row-major, may be a row slice)
    receives C; ``accumulate`` adds into an fp32 ``out``.
    """
    M, K = (a.shape[1], a.shape[0]) if a_mn else a.shape
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    nat.call("nfb_tc_gemm_ex", nat.ptr(a), nat.ptr(b), nat.ptr(out), M, N, K, a.stride(0), b.stride(0),
             out.stride(0), int(out.dtype == torch.float32), int(a_mn), int(b_mn), int(accumulate),
             nat.ptr(status_word(a.device)), nat.stream(a.device))
    return out


def _native_grad_gemms(V: int, H: int, dtype: torch.dtype) -> bool:
    return (os.environ.get("NFB_CE_TC_GRAD_GEMM", "1") != "0" and dtype == torch.bfloat16
            and V % 8 == 0 and H % 8 == 0)


class _CrossEntropyTC(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, ignore_index, chunk_rows):
        M, H = hidden.shape
        V = weight.shape[0]
        dev = hidden.device
        h = hidden if hidden.dtype == torch.bfloat16 else hidden.to(torch.bfloat16)
        w = weight if weight.dtype == torch.bfloat16 else weight.to(torch.bfloat16)
        h = h.contiguous()
        w = w.contiguous()
        tg = targets.contiguous()
        st = status_word(dev)
        count = count_valid(tg, ignore_index)
        n_tiles = int(nat.lib().nfb_ce_tc_tiles(V))
        pmax = torch.empty((M, n_tiles), dtype=torch.float32, device=dev)
        psum = torch.empty((M, n_tiles), dtype=torch.float32, device=dev)
        tlogit = torch.zeros(M, dtype=torch.float32, device=dev)
        lse = torch.empty(M, dtype=torch.float32, device=dev)
        loss_rows = torch.empty(M, dtype=torch.float32, device=dev)
        s = nat.stream(dev)
        nat.call("nfb_ce_tc_stats", nat.ptr(h), h.stride(0), nat.ptr(w), w.stride(0), nat.ptr(tg), M, V, H,
                 nat.ptr(pmax), nat.ptr(psum), nat.ptr(tlogit), nat.ptr(st), s)
        nat.call("nfb_ce_tc_merge", nat.ptr(pmax), nat.ptr(psum), nat.ptr(tlogit), nat.ptr(tg), nat.ptr(count), M, V,
                 ignore_index, nat.ptr(lse), nat.ptr(loss_rows), s)
        d_hidden = torch.empty((M, H), dtype=hidden.dtype, device=dev)
        native_grad = _native_grad_gemms(V, H, hidden.dtype) and h.stride(1) == 1
        # the first chunk's d_W GEMM overwrites, so the native path needs no zero fill
        d_weight = (torch.empty if native_grad else torch.zeros)((V, H), dtype=torch.float32, device=dev)
        for r0 in range(0, M, chunk_rows):
            r1 = min(r0 + chunk_rows, M)
            hc = h[r0:r1]
            dl = torch.empty((r1 - r0, V), dtype=torch.bfloat16, device=dev)
            nat.call("nfb_ce_tc_grad", nat.ptr(hc), hc.stride(0), nat.ptr(w), w.stride(0), nat.ptr(tg[r0:r1]),
                     nat.ptr(lse[r0:r1]), nat.ptr(count), ignore_index, r1 - r0, V, H, nat.ptr(dl), dl.stride(0),
                     nat.ptr(st), s)
            if native_grad:
                # on the CTA-pair core of the linear layers: d_hidden[chunk] = dl @ W (W read as an
                # MN-major B, the input-gradient shape); d_W (+)= dl^T @ h (both MN-major, fp32, the
                # weight-gradient shape, added by TMA reductions)
                _linear.gemm(dl, w, b_mn=True, out=d_hidden[r0:r1])
                _linear.gemm_acc(dl, hc, d_weight, a_mn=True, b_mn=True, accumulate=r0 > 0)
            else:
                d_hidden[r0:r1] = torch.mm(dl, w).to(hidden.dtype)
                d_weight += torch.mm(dl.t(), hc, out_dtype=torch.float32)
            del dl
        ctx.save_for_backward(d_hidden, d_weight)
        ctx.wdtype = weight.dtype
        return loss_rows.sum()

    @staticmethod
    def backward(ctx, g):
        d_hidden, d_weight = ctx.saved_tensors
        return d_hidden * g.to(d_hidden.dtype), (d_weight * g).to(ctx.wdtype), None, None, None


def cross_entropy_tc(hidden, weight, targets, ignore_index: int = -100, chunk_rows: int | None = None):
    """Mean CE over hidden @ weight.T on the tcgen05 path, or None when the shape is unsupported."""
    if not (hidden.is_cuda and nat.HAS_NATIVE) or hidden.dim() != 2:
        return None
    M, H = hidden.shape
    V = weight.shape[0]
    if H % 8 or M == 0 or M >= 2**31 or V >= 2**31:
        return None
    if chunk_rows is None:
        # bound the bf16 dlogits buffer to ~256 MiB
        chunk_rows = max(128, (256 * 2**20) // (2 * V) // 128 * 128)
    return _CrossEntropyTC.apply(hidden, weight, targets, int(ignore_index), int(chunk_rows))


def enable(flag: bool = True) -> None:
    """Route ops.chunked_cross_entropy through the tcgen05 path (default: on unless NFB_CE_TC=0)."""
    register_tc(cross_entropy_tc if flag else None)


enable(os.environ.get("NFB_CE_TC", "1") != "0")

"""Memory-efficient cross entropy for the reasoning head.

Parity: nuvla_forge/kernels/chunked_ce.py:185-208 — ``chunked_cross_entropy(
hidden [M,H], lm_weight [V,H], targets [M], chunk_size=1024, ignore_index=-100,
force_reference=False)`` returns the mean CE over non-ignored tokens, and the
gradient is computed during forward so only parameter-sized gradients survive
to backward (backward just scales them by the upstream scalar).

On the GPU this module is the dispatcher: the tcgen05 path (ops/ce_tc.py,
logits live only in TMEM, online softmax in the GEMM epilogue) when the native
library provides it, else the chunked path below (cuBLAS logit GEMM in fp32 +
the native in-place online-softmax row kernel, csrc/ce_rows.cu). Neither path
synchronises the host: the valid-token count stays on the device.
"""

from __future__ import annotations

import torch

from .. import _native as nat
from .reference import chunked_cross_entropy_ref

_tc_impl = None


def register_tc(fn) -> None:
    global _tc_impl
    _tc_impl = fn


def count_valid(targets: torch.Tensor, ignore_index: int) -> torch.Tensor:
    out = torch.empty(1, dtype=torch.float32, device=targets.device)
    nat.call("nfb_count_valid", nat.ptr(targets), targets.numel(), ignore_index, nat.ptr(out),
             nat.stream(targets.device))
    return out


def _ce_chunk_torch(logits, targets, ignore_index, inv_count):
    """One chunk on the reference path: (sum of scaled row losses, dlogits)."""
    valid = targets != ignore_index
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    safe = torch.where(valid, targets, torch.zeros_like(targets))
    tl = lf.gather(1, safe[:, None]).squeeze(1)
    loss = torch.where(valid, lse - tl, torch.zeros_like(lse)).sum() * inv_count
    p = torch.softmax(lf, dim=-1)
    p[torch.arange(p.shape[0], device=p.device), safe] -= 1.0
    p = p * valid[:, None].to(p.dtype) * inv_count
    return loss, p


class _ChunkedCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, chunk_size, ignore_index, native):
        M, H = hidden.shape
        V = weight.shape[0]
        dev = hidden.device
        d_hidden = torch.empty_like(hidden)
        d_weight = torch.zeros((V, H), dtype=torch.float32, device=dev)
        if native:
            count = count_valid(targets, ignore_index)
            loss_rows = torch.empty(M, dtype=torch.float32, device=dev)
            wlp = weight if weight.dtype in (torch.bfloat16, torch.float16) else weight.to(torch.bfloat16)
            for s in range(0, M, chunk_size):
                e = min(s + chunk_size, M)
                hc = hidden[s:e]
                hlp = hc if hc.dtype == wlp.dtype else hc.to(wlp.dtype)
                logits = torch.mm(hlp, wlp.t(), out_dtype=torch.float32)
                nat.call("nfb_ce_rows", 0, nat.ptr(logits), logits.stride(0), nat.ptr(targets[s:e].contiguous()),
                         e - s, V, ignore_index, nat.ptr(count), nat.ptr(loss_rows[s:e]), nat.stream(dev))
                dl = logits.to(wlp.dtype)
                del logits
                d_hidden[s:e] = torch.mm(dl, wlp).to(hidden.dtype)
                d_weight += torch.mm(dl.t(), hlp, out_dtype=torch.float32)
            loss = loss_rows.sum()
        else:
            n_valid = (targets != ignore_index).sum().clamp(min=1).to(torch.float32)
            inv = 1.0 / n_valid
            loss = torch.zeros((), dtype=torch.float32, device=dev)
            wf = weight.float()
            for s in range(0, M, chunk_size):
                e = min(s + chunk_size, M)
                hf = hidden[s:e].float()
                cl, dl = _ce_chunk_torch(hf @ wf.t(), targets[s:e], ignore_index, inv)
                loss = loss + cl
                d_hidden[s:e] = (dl @ wf).to(hidden.dtype)
                d_weight += dl.t() @ hf
        ctx.save_for_backward(d_hidden, d_weight)
        ctx.wdtype = weight.dtype
        return loss

    @staticmethod
    def backward(ctx, g):
        d_hidden, d_weight = ctx.saved_tensors
        return (d_hidden * g.to(d_hidden.dtype)), (d_weight * g).to(ctx.wdtype), None, None, None, None


def chunked_cross_entropy(hidden: torch.Tensor, lm_weight: torch.Tensor, targets: torch.Tensor,
                          chunk_size: int = 1024, ignore_index: int = -100,
                          force_reference: bool = False) -> torch.Tensor:
    """Mean cross entropy over ``hidden @ lm_weight.T`` without a full [M, V] logit tensor."""
    native = (not force_reference) and nat.HAS_NATIVE and hidden.is_cuda
    if native and _tc_impl is not None:
        out = _tc_impl(hidden, lm_weight, targets, ignore_index)
        if out is not None:
            return out
    return _ChunkedCE.apply(hidden, lm_weight, targets, int(chunk_size), int(ignore_index), native)


__all__ = ["chunked_cross_entropy", "chunked_cross_entropy_ref"]

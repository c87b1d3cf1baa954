"""Attention in the projection-native [B, S, H, D] layout.

``attention(q, k, v, causal)`` takes q [B, S, Hq, D] and k, v [B, L, Hkv, D]
(GQA when Hkv divides Hq) exactly as they come out of a fused qkv projection,
and returns [B, S, Hq, D], which feeds the output projection without a
transpose copy. Parity: the reference calls F.scaled_dot_product_attention on
[B, H, S, D] views (nuvla_forge/model/dit.py:92) and nn.MultiheadAttention
(nuvla_forge/model/nuvla.py:110-112).

Dispatch: the sm_100a flash-attention kernel (csrc/attention.cu) when it is
built and the shape is supported, else PyTorch SDPA, else (CPU or
``force_reference``) the fp32 reference.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _native as nat
from .reference import attention_ref

_native_attention = None


def register_native(fn) -> None:
    """Install the native attention implementation (called by ops.flash_attn)."""
    global _native_attention
    _native_attention = fn


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
              scale: float | None = None, force_reference: bool = False) -> torch.Tensor:
    if force_reference or not q.is_cuda:
        out = attention_ref(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), causal, scale)
        return out.transpose(1, 2)
    if _native_attention is not None and nat.HAS_NATIVE:
        out = _native_attention(q, k, v, causal, scale)
        if out is not None:
            return out
    gqa = k.shape[2] != q.shape[2]
    out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                         is_causal=causal, scale=scale, enable_gqa=gqa)
    return out.transpose(1, 2)

"""Ops: the model's hot operations, native sm_100a kernels with PyTorch references.

Public names mirror the reference's kernel package (nuvla_forge/kernels/__init__.py:8-18)
plus the ops the reference left to PyTorch.
"""

from .._native import HAS_NATIVE
from . import ce_tc  # noqa: F401  (registers the tcgen05 cross-entropy path)
from . import flash_attn  # noqa: F401  (tcgen05 attention forward; opt-in via NFB_ATTN_NATIVE=1)
from .attention import attention
from .chunked_ce import chunked_cross_entropy
from .image import normalise_images, patchify_images
from .norm import add_rmsnorm, fused_adaln_residual_rmsnorm, rmsnorm
from .swiglu import fused_swiglu, swiglu_packed

__all__ = [
    "HAS_NATIVE",
    "add_rmsnorm",
    "attention",
    "chunked_cross_entropy",
    "fused_adaln_residual_rmsnorm",
    "fused_swiglu",
    "normalise_images",
    "patchify_images",
    "rmsnorm",
    "swiglu_packed",
]

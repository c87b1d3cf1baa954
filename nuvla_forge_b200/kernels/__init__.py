"""Kernel API under the reference's module name (nuvla_forge.kernels).

``HAS_NATIVE`` replaces the reference's ``HAS_TRITON`` capability flag; the
three fused ops keep their signatures and ``force_reference`` switch.
"""

from ..ops import HAS_NATIVE, chunked_cross_entropy, fused_adaln_residual_rmsnorm, fused_swiglu
from ..ops import reference  # noqa: F401

__all__ = ["HAS_NATIVE", "chunked_cross_entropy", "fused_adaln_residual_rmsnorm", "fused_swiglu", "reference"]

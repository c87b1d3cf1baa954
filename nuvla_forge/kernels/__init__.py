"""``nuvla_forge.kernels``: the fused ops (native sm_100a kernels) and the capability flag.

``HAS_TRITON`` keeps the reference's name for "the fast path is available"; here it
is the native library's ``HAS_NATIVE``.
"""

from nuvla_forge_b200.kernels import HAS_NATIVE, chunked_cross_entropy, fused_adaln_residual_rmsnorm, fused_swiglu

HAS_TRITON = HAS_NATIVE

__all__ = ["HAS_NATIVE", "HAS_TRITON", "chunked_cross_entropy", "fused_adaln_residual_rmsnorm", "fused_swiglu"]

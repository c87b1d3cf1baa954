"""``nuvla_forge.kernels.adaln_rmsnorm`` (native norm kernels, csrc/norm.cu)."""

from nuvla_forge_b200.ops.norm import fused_adaln_residual_rmsnorm  # noqa: F401

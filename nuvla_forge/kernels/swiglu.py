"""``nuvla_forge.kernels.swiglu`` (native SwiGLU kernels, csrc/swiglu.cu)."""

from nuvla_forge_b200.ops.swiglu import fused_swiglu  # noqa: F401

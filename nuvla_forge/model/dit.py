"""``nuvla_forge.model.dit``."""

from nuvla_forge_b200.models.dit import DiTBlock, TrajectoryDiT  # noqa: F401
from nuvla_forge_b200.models.layers import Attention, RMSNorm, SwiGLUMLP, TimestepEmbedder, modulate  # noqa: F401

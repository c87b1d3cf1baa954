"""``nuvla_forge.model``."""

from nuvla_forge_b200.model import DiTBlock, MultiViewEncoder, NuVLA, NuVLAConfig, TrajectoryDiT  # noqa: F401

__all__ = ["DiTBlock", "MultiViewEncoder", "NuVLA", "NuVLAConfig", "TrajectoryDiT"]

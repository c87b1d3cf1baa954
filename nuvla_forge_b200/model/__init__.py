"""Model API under the reference's module name (nuvla_forge.model)."""

from ..models import DiTBlock, MultiViewEncoder, NuVLA, NuVLAConfig, TrajectoryDiT

__all__ = ["DiTBlock", "MultiViewEncoder", "NuVLA", "NuVLAConfig", "TrajectoryDiT"]

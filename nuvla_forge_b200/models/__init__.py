"""Model definitions: multi-view ViT, VLM backbone, adaLN-Zero trajectory DiT, reasoning head."""

from .dit import DiTBlock, TrajectoryDiT
from .layers import Attention, RMSNorm, SwiGLUMLP, TimestepEmbedder, TransformerBlock
from .nuvla import MultiViewEncoder, NuVLA, NuVLAConfig, SceneQueryPool

__all__ = ["Attention", "DiTBlock", "MultiViewEncoder", "NuVLA", "NuVLAConfig", "RMSNorm", "SceneQueryPool",
           "SwiGLUMLP", "TimestepEmbedder", "TrajectoryDiT", "TransformerBlock"]

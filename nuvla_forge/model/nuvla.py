"""``nuvla_forge.model.nuvla``."""

from nuvla_forge_b200.models.layers import TransformerBlock  # noqa: F401
from nuvla_forge_b200.models.nuvla import MultiViewEncoder, NuVLA, NuVLAConfig  # noqa: F401

"""``nuvla_forge.data.adapters``."""

from nuvla_forge_b200.data.adapters import *  # noqa: F401,F403
from nuvla_forge_b200.data.adapters import REGISTRY, SampleSpec, build_dataset  # noqa: F401

"""``nuvla_forge.data``."""

from nuvla_forge_b200.data import *  # noqa: F401,F403
from nuvla_forge_b200.data import __all__  # noqa: F401

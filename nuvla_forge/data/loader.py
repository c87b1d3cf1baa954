"""``nuvla_forge.data.loader``."""

from nuvla_forge_b200.data.loader import *  # noqa: F401,F403
from nuvla_forge_b200.data.loader import (CudaPrefetcher, LoaderConfig, build_fast_loader,  # noqa: F401
                                          build_naive_loader, describe_environment)

"""``nuvla_forge.kernels.reference``: the pure-PyTorch oracles."""

from nuvla_forge_b200.ops.reference import *  # noqa: F401,F403
from nuvla_forge_b200.ops.reference import (adaln_residual_rmsnorm_ref, chunked_cross_entropy_ref,  # noqa: F401
                                            swiglu_ref)

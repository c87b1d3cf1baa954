"""Reference oracles under the reference's module path (nuvla_forge.kernels.reference)."""

from ..ops.reference import *  # noqa: F401,F403
from ..ops.reference import (adaln_residual_rmsnorm_ref, chunked_cross_entropy_ref,  # noqa: F401
                             swiglu_ref)

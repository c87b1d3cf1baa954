"""The reference's import path, served by nuvla_forge_b200.

Code written against ``nuvla_forge`` (``from nuvla_forge.kernels import
fused_swiglu``, ``python -m nuvla_forge.train --preset optimised``) runs
unchanged on the B200-native implementation: every module below re-exports
the corresponding ``nuvla_forge_b200`` API (parity: nuvla_forge/__init__.py,
nuvla_forge/kernels/__init__.py:8-18).
"""

from nuvla_forge_b200 import __version__  # noqa: F401

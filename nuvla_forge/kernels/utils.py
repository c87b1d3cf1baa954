"""``nuvla_forge.kernels.utils``: capability flags."""

from nuvla_forge_b200._native import HAS_NATIVE  # noqa: F401

HAS_TRITON = HAS_NATIVE

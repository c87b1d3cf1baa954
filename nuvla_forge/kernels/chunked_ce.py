"""``nuvla_forge.kernels.chunked_ce`` (tcgen05 cross entropy, csrc/ce_tc.cu)."""

from nuvla_forge_b200.ops.chunked_ce import chunked_cross_entropy  # noqa: F401

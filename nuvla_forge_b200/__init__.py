"""nuvla_forge_b200: a B200-native (sm_100a) training framework for nuVLA-style driving planners.

Packages: ``ops`` (native kernels + references), ``models``, ``parallel``
(DDP/FSDP runtimes and fused NVLink collectives), ``optim``, ``data``,
``utils``; ``train`` is the training entry point.
"""

__version__ = "0.1.0"

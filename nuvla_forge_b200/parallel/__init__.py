"""Parallel runtimes: process-group bootstrap, symmetric memory, DDP and FSDP with fused NVLink collectives."""

from .ddp import DistributedDataParallel
from .dist import DistInfo, max_over_ranks, setup_distributed, teardown_distributed
from .flat import FlatParamSpace

__all__ = ["DistInfo", "DistributedDataParallel", "FlatParamSpace", "max_over_ranks", "setup_distributed",
           "teardown_distributed"]

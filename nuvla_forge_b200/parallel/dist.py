"""Process-group bootstrap: one process per GPU, NCCL on GPUs, gloo on CPU.

Parity: nuvla_forge/train.py:41-49 (setup_distributed). The reference
hard-codes ``nccl`` and therefore cannot run under torchrun on CPU; here the
backend follows the device, every group gets a bounded timeout (so ranks that
wait for a dead peer end with an error), and rendezvous defaults to
127.0.0.1.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    device: torch.device = torch.device("cpu")
    backend: str = "none"

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def setup_distributed(backend: str | None = None, timeout_s: float | None = None) -> DistInfo:
    """Initialise the default process group from torchrun's environment (no-op without RANK)."""
    cuda = torch.cuda.is_available()
    if "RANK" not in os.environ:
        dev = torch.device("cuda:0" if cuda else "cpu")
        if cuda:
            torch.cuda.set_device(0)
        return DistInfo(0, 1, 0, dev, "none")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if cuda:
        torch.cuda.set_device(local)
    backend = backend or ("nccl" if cuda else "gloo")
    timeout = datetime.timedelta(seconds=timeout_s or float(os.environ.get("NFB_PG_TIMEOUT_S", "600")))
    if not dist.is_initialized():
        kw = {"backend": backend, "timeout": timeout}
        if cuda and backend == "nccl":
            kw["device_id"] = torch.device(f"cuda:{local}")
        dist.init_process_group(**kw)
    dev = torch.device(f"cuda:{local}" if cuda else "cpu")
    return DistInfo(dist.get_rank(), dist.get_world_size(), local, dev, backend)


def teardown_distributed() -> None:
    if dist.is_available() and dist.is_initialized():
        try:
            dist.barrier()
        finally:
            dist.destroy_process_group()


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """Max of a host scalar over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    dev = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                     and dist.get_backend() == "nccl" else torch.device("cpu"))
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())

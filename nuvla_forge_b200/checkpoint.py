"""Checkpoint save / resume.

The reference never saves (no torch.save or state_dict use anywhere); the
format honoured is the plain ``nn.Module.state_dict()`` of the model, so a
checkpoint written here loads into the reference's ``NuVLA`` with
``load_state_dict`` (for the default config). File layout::

    {"model": {name: fp32 tensor, ...},        # full, unsharded, reference key names
     "optim": {...}, "step": int, "rng": {...}, "rng_per_rank": [{...}, ...], "config": {...}}

Every rank's RNG state is saved (ranks draw different noise: the trainer seeds
rank r with seed + r), and each rank restores its own on resume; with a
different world size a rank without an entry is reseeded from (seed, rank, step).

Model tensors come from the fp32 master weights (not the bf16 compute copy).
Under FSDP the shards are gathered to rank 0, which writes the file.
"""

from __future__ import annotations

import os
import random
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist


def _fp32_state_dict(module: torch.nn.Module, master_views: dict[int, torch.Tensor]) -> dict:
    """module.state_dict() with every parameter replaced by its fp32 master copy."""
    saved = {}
    try:
        for p in module.parameters():
            mv = master_views.get(id(p))
            if mv is not None:
                saved[id(p)] = p.data
                p.data = mv
        sd = module.state_dict()
        return {k: v.detach().to(torch.float32).cpu().clone() for k, v in sd.items()}
    finally:
        for p in module.parameters():
            if id(p) in saved:
                p.data = saved[id(p)]


def rng_state() -> dict:
    st = {"torch": torch.get_rng_state(), "numpy": np.random.get_state(), "python": random.getstate()}
    if torch.cuda.is_available():
        st["cuda"] = torch.cuda.get_rng_state()
    return st


def set_rng_state(st: dict) -> None:
    torch.set_rng_state(st["torch"])
    np.random.set_state(st["numpy"])
    random.setstate(st["python"])
    if "cuda" in st and torch.cuda.is_available():
        torch.cuda.set_rng_state(st["cuda"])


def model_state_dict(wrapper) -> dict:
    """Full fp32 reference-format state dict (collective under FSDP: call on every rank)."""
    if hasattr(wrapper, "full_master_views"):
        views = wrapper.full_master_views()
        return _fp32_state_dict(wrapper.module, views) if views is not None else {}
    space = wrapper.space
    views = {id(s.param): space.master[s.start: s.start + s.numel].view(s.shape) for s in space.segments}
    return _fp32_state_dict(wrapper.module, views)


def save_checkpoint(path: str | Path, wrapper, optimizer, step: int, config: dict | None = None) -> None:
    sd = model_state_dict(wrapper)
    optim_sd = optimizer.state_dict()
    if hasattr(wrapper, "gather_optimizer_state"):
        optim_sd = wrapper.gather_optimizer_state(optimizer)
    rank = dist.get_rank() if dist.is_initialized() else 0
    mine = rng_state()
    if dist.is_initialized() and dist.get_world_size() > 1:
        per_rank = [None] * dist.get_world_size()
        dist.all_gather_object(per_rank, mine)
    else:
        per_rank = [mine]
    if rank == 0:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(path.suffix + ".tmp")
        torch.save({"model": sd, "optim": optim_sd, "step": int(step), "rng": mine, "rng_per_rank": per_rank,
                    "config": config or {}}, tmp)
        os.replace(tmp, path)
    if dist.is_initialized():
        dist.barrier()


def restore_rng(ck: dict, rank: int, world: int, seed: int = 1234) -> str:
    """Restore this rank's RNG from checkpoint ``ck``. Returns "own", "reseeded" or "none"."""
    per_rank = ck.get("rng_per_rank")
    try:
        if per_rank and len(per_rank) == world and per_rank[rank] is not None:
            set_rng_state(per_rank[rank])
            return "own"
        if per_rank or ck.get("rng"):
            # the world size changed: keep the Python/NumPy streams of rank 0, give torch a distinct seed
            set_rng_state((per_rank or [ck["rng"]])[0])
            torch.manual_seed(seed + rank + 1000003 * int(ck.get("step", 0)))
            return "reseeded"
    except Exception:  # noqa: BLE001 - RNG layout differs across versions: not fatal
        pass
    return "none"


def load_checkpoint(path: str | Path, wrapper, optimizer=None) -> int:
    ck = torch.load(path, map_location="cpu", weights_only=False)
    if hasattr(wrapper, "load_full_state_dict"):
        wrapper.load_full_state_dict(ck["model"])
        if optimizer is not None and ck.get("optim"):
            wrapper.load_optimizer_state(optimizer, ck["optim"])
    else:
        _load_into_space(wrapper, ck["model"])
        if optimizer is not None and ck.get("optim"):
            optimizer.load_state_dict(ck["optim"])
    rank = dist.get_rank() if dist.is_initialized() else 0
    world = dist.get_world_size() if dist.is_initialized() else 1
    restore_rng(ck, rank, world)
    return int(ck.get("step", 0))


def _load_into_space(wrapper, sd: dict) -> None:
    """Load a reference-format state dict into the module, then refresh the flat master copy."""
    module = wrapper.module
    space = wrapper.space
    # load into fp32 temporaries bound to the master views so nothing is rounded
    saved = {}
    for s in space.segments:
        saved[id(s.param)] = s.param.data
        s.param.data = space.master[s.start: s.start + s.numel].view(s.shape)
    try:
        module.load_state_dict(sd, strict=True)
    finally:
        for s in space.segments:
            s.param.data = saved[id(s.param)]
    space.sync_params_from_master()

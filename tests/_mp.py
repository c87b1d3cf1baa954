"""Spawn helpers for multi-process CPU (gloo) tests."""

import datetime
import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _entry(rank, world, port, fn, q, args, timeout_s, backend="gloo", env=None):
    import sys

    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    os.environ.update(env or {})
    try:
        kw = {}
        if backend == "nccl":
            import torch

            torch.cuda.set_device(rank)
            kw["device_id"] = torch.device(f"cuda:{rank}")
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
        res = fn(rank, world, *args)
        q.put((rank, "ok", _pack(res)))
    except BaseException as exc:  # noqa: BLE001 - report to the parent
        q.put((rank, "err", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}"))
    finally:
        try:
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _pack(obj):
    """Tensors -> numpy (a child may exit before the parent unpickles shared-memory tensors)."""
    import torch

    if isinstance(obj, torch.Tensor):
        t = obj.detach().cpu()
        return ("__tensor__", str(t.dtype), t.float().numpy() if t.dtype == torch.bfloat16 else t.numpy())
    if isinstance(obj, dict):
        return {k: _pack(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_pack(v) for v in obj)
    return obj


def _unpack(obj):
    import torch

    if isinstance(obj, tuple) and len(obj) == 3 and obj[0] == "__tensor__":
        t = torch.from_numpy(obj[2])
        return t.to(torch.bfloat16) if obj[1] == "torch.bfloat16" else t
    if isinstance(obj, dict):
        return {k: _unpack(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_unpack(v) for v in obj)
    return obj


def run_ranks(fn, world: int = 2, args=(), timeout_s: float = 60.0, join_s: float = 120.0, backend: str = "gloo",
              env: dict | None = None) -> dict:
    """Run fn(rank, world, *args) on `world` ranks (gloo on CPU, or nccl with rank r on cuda:r).

    Returns {rank: (status, result)}."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, q, args, timeout_s, backend, env))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    import queue
    import time

    deadline = time.time() + join_s
    while len(out) < world and time.time() < deadline:
        try:
            r, st, res = q.get(timeout=1.0)
            out[r] = (st, _unpack(res))
        except queue.Empty:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=5)
        if p.is_alive():
            p.kill()
            p.join()
    return out

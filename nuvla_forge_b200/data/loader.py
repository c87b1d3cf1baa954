"""Loaders, collate, the CUDA prefetcher and the synthetic pinned-batch source.

Parity: nuvla_forge/data/loader.py:60-255 (LoaderConfig, hash tokenizer,
collate, build_naive_loader, build_fast_loader, CudaPrefetcher,
normalise_images, write_shards, describe_environment). Differences:

* Images stay uint8 HWC [B, V*F, H, W, 3]: the host never transposes them
  (the reference permuted every batch to CHW on the CPU); the device-side
  patchify kernel reads HWC directly.
* When a record carries ``instruction``/``reasoning`` ids, the text is their
  concatenation and the targets are next-token ids over the reasoning span
  (-100 elsewhere). Otherwise the reference's hash tokenizer and its
  "targets = inputs" convention are kept.
* ``SyntheticBatchSource`` produces whole batches straight into a ring of
  pinned host buffers with the native generator (no per-sample Python, no
  collate copies), which is what the throughput benchmarks feed from.
"""

from __future__ import annotations

import io
import os
import tarfile
import threading
import zlib
from collections.abc import Iterator
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch
from torch.utils.data import DataLoader

from ..ops.image import normalise_images as _normalise_native
from .adapters import SampleSpec, random_views, unicycle_trajectory

try:
    import webdataset  # noqa: F401
    HAS_WDS = True
except Exception:  # noqa: BLE001 - optional dependency probe
    HAS_WDS = False

try:
    from nvidia.dali import pipeline_def  # noqa: F401
    HAS_DALI = True
except Exception:  # noqa: BLE001 - optional dependency probe
    HAS_DALI = False


@dataclass
class LoaderConfig:
    batch_size: int = 8
    num_workers: int = 8
    prefetch_factor: int = 4
    pin_memory: bool = True
    persistent_workers: bool = True
    drop_last: bool = True
    max_text_len: int = 64
    vocab_size: int = 32000


def _hash_tokenize(text: str, max_len: int, vocab_size: int) -> np.ndarray:
    """Deterministic word-hash ids in [1, vocab) padded with -100 (crc32, not the salted hash())."""
    ids = np.full(max_len, -100, dtype=np.int64)
    for i, word in enumerate(text.lower().split()[:max_len]):
        ids[i] = zlib.crc32(word.encode()) % (vocab_size - 1) + 1
    return ids


def next_token_targets(instruction: np.ndarray, reasoning: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """tokens = [instr ; reasoning]; target[t] = tokens[t+1] on the reasoning span, -100 elsewhere."""
    tokens = np.concatenate([instruction, reasoning])
    targets = np.full_like(tokens, -100)
    li, lr = len(instruction), len(reasoning)
    if lr:
        start = max(li - 1, 0)
        targets[start: li + lr - 1] = tokens[start + 1: li + lr]
    return tokens, targets


def collate(batch, cfg: LoaderConfig):
    images = torch.from_numpy(np.stack([b["images"] for b in batch]))   # [B, V*F, H, W, 3] uint8
    trajectory = torch.from_numpy(np.stack([b["trajectory"] for b in batch]))
    if "reasoning" in batch[0]:
        pairs = [next_token_targets(b["instruction"], b["reasoning"]) for b in batch]
        tokens = torch.from_numpy(np.stack([p[0] for p in pairs]))
        targets = torch.from_numpy(np.stack([p[1] for p in pairs]))
    else:
        text = np.stack([_hash_tokenize(f"{b['question']} {b['answer']}", cfg.max_text_len, cfg.vocab_size)
                         for b in batch])
        tokens = torch.from_numpy(np.where(text < 0, 0, text))
        targets = torch.from_numpy(text)
    return {"images": images, "trajectory": trajectory, "text_tokens": tokens, "text_targets": targets}


class _Collate:
    """Picklable collate (DataLoader workers)."""

    def __init__(self, cfg: LoaderConfig):
        self.cfg = cfg

    def __call__(self, batch):
        return collate(batch, self.cfg)


def build_naive_loader(dataset, cfg: LoaderConfig, sampler=None) -> DataLoader:
    """Deliberately untuned baseline: 2 workers, no pinning (reference: loader.py:110-121)."""
    return DataLoader(dataset, batch_size=cfg.batch_size, num_workers=2, shuffle=sampler is None, sampler=sampler,
                      pin_memory=False, drop_last=cfg.drop_last, collate_fn=_Collate(cfg))


def build_fast_loader(dataset, cfg: LoaderConfig, sampler=None) -> DataLoader:
    """Tuned: worker count, prefetch depth, pinning, persistent workers (reference: loader.py:124-138)."""
    kw = dict(batch_size=cfg.batch_size, num_workers=cfg.num_workers, shuffle=sampler is None, sampler=sampler,
              pin_memory=cfg.pin_memory and torch.cuda.is_available(), drop_last=cfg.drop_last,
              collate_fn=_Collate(cfg))
    if cfg.num_workers > 0:
        kw["prefetch_factor"] = cfg.prefetch_factor
        kw["persistent_workers"] = cfg.persistent_workers
    return DataLoader(dataset, **kw)


class CudaPrefetcher:
    """Overlaps the host->device copy of batch N+1 with the compute of batch N.

    Parity: nuvla_forge/data/loader.py:141-183 (side stream, wait_stream,
    record_stream so the caching allocator does not recycle in-flight buffers).
    """

    def __init__(self, loader, device):
        self.loader = loader
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device)

    def __len__(self):
        return len(self.loader)

    def _to_device(self, batch):
        if batch is None:
            return None
        with torch.cuda.stream(self.stream):
            return {k: v.to(self.device, non_blocking=True) if isinstance(v, torch.Tensor) else v
                    for k, v in batch.items()}

    def __iter__(self) -> Iterator[dict]:
        it = iter(self.loader)
        nxt = self._to_device(next(it, None))
        while nxt is not None:
            cur_stream = torch.cuda.current_stream(self.device)
            cur_stream.wait_stream(self.stream)
            cur = nxt
            for v in cur.values():
                if isinstance(v, torch.Tensor):
                    v.record_stream(cur_stream)
            nxt = self._to_device(next(it, None))
            yield cur


class SyntheticBatchSource:
    """Whole synthetic batches generated straight into pinned host memory.

    A background thread fills up to ``depth`` batches ahead; images come from
    the native multithreaded generator, deterministic in (seed, global sample
    index), so data-parallel ranks draw disjoint samples by passing
    ``rank``/``world``. Every batch gets fresh buffers from PyTorch's caching
    pinned-memory allocator, which keeps a block out of reuse until the
    non-blocking device copies issued from it have completed; so consumers may
    copy whenever they like and simply drop the batch afterwards.
    """

    def __init__(self, spec: SampleSpec, batch_size: int, seed: int = 0, rank: int = 0, world: int = 1,
                 depth: int = 4, threads: int | None = None, pin: bool | None = None, n_batches: int | None = None,
                 copy_stream=None):
        self.spec = spec
        self.bs = batch_size
        self.seed = seed
        self.rank, self.world = rank, world
        self.depth = max(1, depth)
        self.threads = threads or max(1, min(8, (os.cpu_count() or 2) // max(world, 1)))
        self.pin = torch.cuda.is_available() if pin is None else pin
        self.n_batches = n_batches
        L = (spec.n_instruction + spec.n_reasoning) or spec.max_text_len
        self._shapes = {
            "images": ((batch_size, spec.n_images, spec.image_size, spec.image_size, 3), torch.uint8),
            "trajectory": ((batch_size, spec.horizon, spec.traj_dim), torch.float32),
            "text_tokens": ((batch_size, L), torch.int64),
            "text_targets": ((batch_size, L), torch.int64),
        }

    def _alloc(self):
        return {k: torch.empty(s, dtype=d, pin_memory=self.pin) for k, (s, d) in self._shapes.items()}

    def bytes_per_batch(self) -> int:
        return sum(int(np.prod(s)) * torch.empty((), dtype=d).element_size() for s, d in self._shapes.values())

    def fill(self, buf: dict, batch_index: int) -> dict:
        sp = self.spec
        imgs = buf["images"].numpy()
        for i in range(self.bs):
            gidx = (batch_index * self.world + self.rank) * self.bs + i
            random_views(sp, self.seed, gidx, out=imgs[i], threads=self.threads)
            rng = np.random.default_rng((self.seed, gidx))
            buf["trajectory"][i] = torch.from_numpy(unicycle_trajectory(sp, rng))
            if sp.n_instruction or sp.n_reasoning:
                ins = rng.integers(0, sp.vocab_size, sp.n_instruction, dtype=np.int64)
                rea = rng.integers(0, sp.vocab_size, sp.n_reasoning, dtype=np.int64)
                tok, tgt = next_token_targets(ins, rea)
            else:
                tgt = rng.integers(1, sp.vocab_size, sp.max_text_len, dtype=np.int64)
                tok = tgt
            buf["text_tokens"][i] = torch.from_numpy(tok)
            buf["text_targets"][i] = torch.from_numpy(tgt)
        return buf

    def batch(self, batch_index: int) -> dict:
        """Generate batch ``batch_index`` synchronously."""
        return self.fill(self._alloc(), batch_index)

    def __iter__(self) -> Iterator[dict]:
        import queue

        q: queue.Queue = queue.Queue(maxsize=self.depth)
        done = threading.Event()

        def producer():
            k = 0
            while not done.is_set() and (self.n_batches is None or k < self.n_batches):
                b = self.batch(k)
                while not done.is_set():
                    try:
                        q.put(b, timeout=0.1)
                        break
                    except queue.Full:
                        continue
                k += 1
            q.put(None)

        th = threading.Thread(target=producer, daemon=True)
        th.start()
        try:
            while True:
                b = q.get()
                if b is None:
                    return
                yield b
        finally:
            done.set()


def normalise_images(images: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """uint8 [B, V, 3, H, W] -> ImageNet-normalised ``dtype`` on the device (one native kernel)."""
    return _normalise_native(images, dtype)


def write_shards(dataset, out_dir: str | Path, samples_per_shard: int = 512, limit: int | None = None) -> list[Path]:
    """Pack records into tar shards of ``<key>.images.npy``, ``.trajectory.npy``, ``.question.txt``, ``.answer.txt``."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    n = min(len(dataset), limit or len(dataset))
    shards: list[Path] = []
    tar = None
    try:
        for i in range(n):
            if i % samples_per_shard == 0:
                if tar is not None:
                    tar.close()
                path = out_dir / f"shard-{len(shards):05d}.tar"
                shards.append(path)
                tar = tarfile.open(path, "w")  # noqa: SIM115 - closed explicitly across iterations
            rec = dataset[i]
            key = f"{i:08d}"
            for name, arr in (("images.npy", rec["images"]), ("trajectory.npy", rec["trajectory"])):
                buf = io.BytesIO()
                np.save(buf, arr)
                info = tarfile.TarInfo(f"{key}.{name}")
                info.size = buf.tell()
                buf.seek(0)
                tar.addfile(info, buf)
            for name, text in (("question.txt", rec["question"]), ("answer.txt", rec["answer"])):
                data = text.encode()
                info = tarfile.TarInfo(f"{key}.{name}")
                info.size = len(data)
                tar.addfile(info, io.BytesIO(data))
    finally:
        if tar is not None:
            tar.close()
    return shards


class ShardDataset(torch.utils.data.Dataset):
    """Reads the shards ``write_shards`` wrote (the reference has a writer but no reader)."""

    def __init__(self, shards: list[str | Path]):
        self.items: list[tuple[Path, str]] = []
        for p in shards:
            with tarfile.open(p) as t:
                keys = sorted({m.name.split(".")[0] for m in t.getmembers()})
            self.items += [(Path(p), k) for k in keys]

    def __len__(self):
        return len(self.items)

    def __getitem__(self, idx):
        path, key = self.items[idx]
        with tarfile.open(path) as t:
            def rd(name):
                return t.extractfile(f"{key}.{name}").read()
            return {"images": np.load(io.BytesIO(rd("images.npy"))),
                    "trajectory": np.load(io.BytesIO(rd("trajectory.npy"))),
                    "question": rd("question.txt").decode(), "answer": rd("answer.txt").decode(),
                    "sample_id": key}


def describe_environment() -> dict:
    return {"cpu_count": os.cpu_count(), "has_dali": HAS_DALI, "has_webdataset": HAS_WDS,
            "torch_threads": torch.get_num_threads()}

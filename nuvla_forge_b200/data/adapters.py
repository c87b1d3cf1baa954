"""Dataset adapters behind one record schema.

Parity: nuvla_forge/data/adapters.py:1-291. Every adapter yields::

    {"images": uint8 [V*F, H, W, 3], "trajectory": float32 [horizon, traj_dim],
     "question": str, "answer": str, "sample_id": str}

and optionally pre-tokenised ``instruction`` / ``reasoning`` int64 arrays (the
synthetic BASELINE datasets draw token ids uniformly, as the configs specify).

``SampleSpec`` gains ``n_frames`` (views x frames are stored view-major),
``traj_dim`` (2 = (x, y) as in the reference, 3 = (x, y, heading)) and the
unicycle parameters (the BASELINE configs use speed ~ U[0, 15] m/s and yaw
rate ~ N(0, 0.1) rad/s; the reference used U[2, 14] and N(0, 0.12)).

Real-data adapters (DriveLM-nuScenes, nuscenes-qa-mini, nuReasoning) keep the
reference's layouts and error messages; they need local files or the
``datasets`` package, neither of which a synthetic benchmark touches.
"""

from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any, ClassVar

import numpy as np
from torch.utils.data import Dataset


@dataclass
class SampleSpec:
    n_views: int = 6
    image_size: int = 224
    horizon: int = 6
    max_text_len: int = 64
    n_frames: int = 1
    traj_dim: int = 2
    speed_range: tuple = (2.0, 14.0)
    yaw_rate_std: float = 0.12
    dt: float = 0.5
    n_instruction: int = 0
    n_reasoning: int = 0
    vocab_size: int = 32000

    @property
    def n_images(self) -> int:
        return self.n_views * self.n_frames

    @staticmethod
    def for_model(cfg) -> "SampleSpec":
        """The data spec matching a NuVLAConfig (BASELINE kinematics for BASELINE presets)."""
        baseline = cfg.backbone_over_images
        return SampleSpec(
            n_views=cfg.n_views, image_size=cfg.image_size, horizon=cfg.horizon, max_text_len=cfg.max_text_len,
            n_frames=cfg.n_frames, traj_dim=cfg.traj_dim,
            speed_range=(0.0, 15.0) if baseline else (2.0, 14.0), yaw_rate_std=0.1 if baseline else 0.12,
            n_instruction=cfg.n_instruction, n_reasoning=cfg.n_reasoning, vocab_size=cfg.vocab_size,
        )


def unicycle_trajectory(spec: SampleSpec, rng: np.random.Generator) -> np.ndarray:
    """Constant speed / yaw-rate rollout; returns [horizon, traj_dim] (x, y[, heading])."""
    speed = rng.uniform(*spec.speed_range)
    yaw_rate = rng.normal(0.0, spec.yaw_rate_std)
    x = y = yaw = 0.0
    out = np.zeros((spec.horizon, spec.traj_dim), dtype=np.float32)
    for i in range(spec.horizon):
        yaw += yaw_rate * spec.dt
        x += speed * spec.dt * np.cos(yaw)
        y += speed * spec.dt * np.sin(yaw)
        row = (x, y, yaw)[: spec.traj_dim]
        out[i, : len(row)] = row
    return out


_synth_lib = None


def _native_fill():
    global _synth_lib
    if _synth_lib is None:
        try:
            from .._build import lib_path
            lib = ctypes.CDLL(str(lib_path()))
            fn = lib.nfb_synth_fill_u8
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int]
            _synth_lib = fn
        except Exception:  # noqa: BLE001 - library not built: numpy fallback
            _synth_lib = False
    return _synth_lib or None


def random_views(spec: SampleSpec, seed: int, idx: int, out: np.ndarray | None = None,
                 threads: int = 1) -> np.ndarray:
    """uint8 [V*F, H, W, 3] uniform in [0, 255], deterministic in (seed, idx)."""
    shape = (spec.n_images, spec.image_size, spec.image_size, 3)
    if out is None:
        out = np.empty(shape, dtype=np.uint8)
    fill = _native_fill()
    if fill is not None and out.flags["C_CONTIGUOUS"]:
        fill(out.ctypes.data, out.size, seed & (2**64 - 1), idx, threads)
    else:
        out[...] = np.random.default_rng((seed, idx)).integers(0, 256, shape, dtype=np.uint8)
    return out


class BaseDrivingDataset(Dataset):
    def __init__(self, spec: SampleSpec, synthetic_trajectory: bool = True, seed: int = 0):
        self.spec = spec
        self.synthetic_trajectory = synthetic_trajectory
        self._seed = seed

    def _rng(self, idx: int) -> np.random.Generator:
        return np.random.default_rng(self._seed + idx)


class SyntheticDriving(BaseDrivingDataset):
    """Synthetic samples with the configured shapes; no downloads (reference: adapters.py:88-107)."""

    def __init__(self, n: int = 4096, spec: SampleSpec | None = None, **kw):
        super().__init__(spec or SampleSpec(), **kw)
        self.n = n

    def __len__(self):
        return self.n

    def __getitem__(self, idx):
        rng = self._rng(idx)
        rec = {
            "images": random_views(self.spec, self._seed, idx),
            "trajectory": unicycle_trajectory(self.spec, rng),
            "question": "what should the ego vehicle do next?",
            "answer": "proceed with caution",
            "sample_id": f"synth-{idx:06d}",
        }
        sp = self.spec
        if sp.n_instruction or sp.n_reasoning:
            rec["instruction"] = rng.integers(0, sp.vocab_size, sp.n_instruction, dtype=np.int64)
            rec["reasoning"] = rng.integers(0, sp.vocab_size, sp.n_reasoning, dtype=np.int64)
        return rec


class DriveLMNuScenes(BaseDrivingDataset):
    """DriveLM-nuScenes QA over nuScenes keyframes (reference: adapters.py:110-187).

    Layout: ``root/v1_0_train_nus.json`` and ``root/nuscenes/samples/<CAM_*>/*.jpg``.
    """

    CAMERAS: ClassVar[list[str]] = ["CAM_FRONT", "CAM_FRONT_RIGHT", "CAM_FRONT_LEFT",
                                    "CAM_BACK", "CAM_BACK_LEFT", "CAM_BACK_RIGHT"]

    def __init__(self, root: str | Path, spec: SampleSpec | None = None, **kw):
        super().__init__(spec or SampleSpec(), **kw)
        self.root = Path(root)
        qa = self.root / "v1_0_train_nus.json"
        if not qa.exists():
            raise FileNotFoundError(
                f"{qa} not found. Fetch it with:\n  huggingface-cli download OpenDriveLab/DriveLM "
                f"--repo-type dataset --local-dir {self.root}")
        with open(qa) as f:
            self.records = self._flatten(json.load(f))

    @staticmethod
    def _flatten(raw: dict[str, Any]) -> list[dict[str, Any]]:
        recs = []
        for scene_token, scene in raw.items():
            for frame_token, frame in scene.get("key_frames", {}).items():
                paths = frame.get("image_paths", {})
                for category, qas in frame.get("QA", {}).items():
                    for qa in qas:
                        recs.append({"scene": scene_token, "frame": frame_token, "paths": paths,
                                     "question": qa.get("Q", ""), "answer": qa.get("A", ""),
                                     "category": category})
        return recs

    def __len__(self):
        return len(self.records)

    def _load_view(self, rel):
        from PIL import Image
        size = self.spec.image_size
        full = self.root / rel if rel else None
        if full is not None and full.exists():
            return np.asarray(Image.open(full).convert("RGB").resize((size, size)), dtype=np.uint8)
        return np.zeros((size, size, 3), dtype=np.uint8)

    def __getitem__(self, idx):
        rec = self.records[idx]
        views = [self._load_view(rec["paths"].get(cam)) for cam in self.CAMERAS[: self.spec.n_views]]
        views = [v for v in views for _ in range(self.spec.n_frames)]
        return {"images": np.stack(views), "trajectory": unicycle_trajectory(self.spec, self._rng(idx)),
                "question": rec["question"], "answer": rec["answer"],
                "sample_id": f"{rec['scene']}/{rec['frame']}/{idx}"}


def _hf_views(rec, spec: SampleSpec, upper: bool = False) -> np.ndarray:
    size = spec.image_size
    keys = sorted(k for k in rec if (k.upper() if upper else k).startswith("CAM"))
    views = [np.asarray(rec[k].convert("RGB").resize((size, size)), dtype=np.uint8)
             for k in keys if hasattr(rec[k], "convert")]
    while len(views) < spec.n_views:
        views.append(np.zeros((size, size, 3), dtype=np.uint8))
    views = views[: spec.n_views]
    return np.stack([v for v in views for _ in range(spec.n_frames)])


class NuScenesQAMini(BaseDrivingDataset):
    """``KevinNotSmile/nuscenes-qa-mini`` through ``datasets`` (reference: adapters.py:190-227)."""

    def __init__(self, split: str = "train", config: str = "day", spec: SampleSpec | None = None, **kw):
        super().__init__(spec or SampleSpec(), **kw)
        from datasets import load_dataset
        self.ds = load_dataset("KevinNotSmile/nuscenes-qa-mini", config, split=split)

    def __len__(self):
        return len(self.ds)

    def __getitem__(self, idx):
        rec = self.ds[idx]
        return {"images": _hf_views(rec, self.spec), "trajectory": unicycle_trajectory(self.spec, self._rng(idx)),
                "question": str(rec.get("question", "")), "answer": str(rec.get("answer", "")),
                "sample_id": f"nqa-{idx:06d}"}


class NuReasoning(BaseDrivingDataset):
    """Motional nuReasoning (gated on the Hub, or local parquet) (reference: adapters.py:230-277)."""

    def __init__(self, root: str | Path | None = None, split: str = "train", spec: SampleSpec | None = None, **kw):
        super().__init__(spec or SampleSpec(), **kw)
        from datasets import load_dataset
        if root and Path(root).exists():
            self.ds = load_dataset("parquet", data_dir=str(root), split=split)
        else:
            self.ds = load_dataset("qixuewei/nuReasoning", split=split, token=os.environ.get("HF_TOKEN"))

    def __len__(self):
        return len(self.ds)

    def __getitem__(self, idx):
        rec = self.ds[idx]
        traj = rec.get("ego_future") or rec.get("trajectory")
        if traj is not None:
            t = np.zeros((self.spec.horizon, self.spec.traj_dim), dtype=np.float32)
            a = np.asarray(traj, dtype=np.float32)[: self.spec.horizon, : self.spec.traj_dim]
            t[: a.shape[0], : a.shape[1]] = a
        else:
            t = unicycle_trajectory(self.spec, self._rng(idx))
        return {"images": _hf_views(rec, self.spec, upper=True), "trajectory": t,
                "question": str(rec.get("question", "")),
                "answer": str(rec.get("answer", rec.get("reasoning", ""))),
                "sample_id": str(rec.get("sample_token", idx))}


REGISTRY = {
    "synthetic": SyntheticDriving,
    "drivelm": DriveLMNuScenes,
    "nuscenes-qa-mini": NuScenesQAMini,
    "nureasoning": NuReasoning,
}


def build_dataset(name: str, **kwargs) -> BaseDrivingDataset:
    if name not in REGISTRY:
        raise KeyError(f"unknown dataset {name!r}; have {sorted(REGISTRY)}")
    return REGISTRY[name](**kwargs)

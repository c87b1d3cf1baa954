"""On-device uint8 image preparation (native kernels in csrc/image.cu).

Parity: nuvla_forge/data/loader.py:186-196 (``normalise_images``). The
reference runs ~4 eager kernels and two host->device constructions per call;
here it is one launch with the per-channel constants folded into an affine
``v * scale[c] + bias[c]``. ``patchify_images`` additionally cuts the HWC frames
into normalised (c, ky, kx) patch rows that feed the patch-embedding GEMM
directly, so neither the host nor the device ever materialises a
channels-first float image.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _native as nat
from .reference import IMAGENET_MEAN, IMAGENET_STD, normalise_images_ref, patchify_ref


def _f3(vals) -> ctypes.Array:
    return (ctypes.c_float * 3)(*[float(v) for v in vals])


def normalise_images(images: torch.Tensor, dtype=torch.bfloat16, mean=IMAGENET_MEAN, std=IMAGENET_STD,
                     force_reference: bool = False) -> torch.Tensor:
    """uint8 [..., 3, H, W] -> (v/255 - mean[c]) / std[c] in ``dtype`` (same layout)."""
    if (force_reference or not nat.HAS_NATIVE or not images.is_cuda or images.dtype != torch.uint8
            or dtype not in nat.DT):
        return normalise_images_ref(images, dtype, mean, std)
    x = images.contiguous()
    out = torch.empty(x.shape, dtype=dtype, device=x.device)
    hw = x.shape[-1] * x.shape[-2]
    nat.call("nfb_image_normalize", nat.dtype_code(dtype), nat.ptr(x), nat.ptr(out), x.numel(), hw,
             ctypes.cast(_f3(mean), ctypes.c_void_p), ctypes.cast(_f3(std), ctypes.c_void_p), nat.stream(x.device))
    return out


def patch_kpad(patch: int) -> int:
    k = 3 * patch * patch
    return (k + 7) // 8 * 8


def patchify_images(images_hwc: torch.Tensor, patch: int, dtype=torch.bfloat16, kpad: int | None = None,
                    mean=IMAGENET_MEAN, std=IMAGENET_STD, force_reference: bool = False) -> torch.Tensor:
    """uint8 [n, H, W, 3] -> normalised patch rows [n, (H/p)*(W/p), kpad], (c, ky, kx) order."""
    kpad = kpad or patch_kpad(patch)
    if (force_reference or not nat.HAS_NATIVE or not images_hwc.is_cuda or dtype not in (torch.bfloat16,
                                                                                       torch.float16)):
        return patchify_ref(images_hwc, patch, kpad, dtype, mean, std)
    x = images_hwc.contiguous()
    n, H, W, _ = x.shape
    out = torch.empty((n, (H // patch) * (W // patch), kpad), dtype=dtype, device=x.device)
    nat.call("nfb_image_patchify", nat.dtype_code(dtype), nat.ptr(x), nat.ptr(out), n, H, W, patch, kpad,
             ctypes.cast(_f3(mean), ctypes.c_void_p), ctypes.cast(_f3(std), ctypes.c_void_p), nat.stream(x.device))
    return out

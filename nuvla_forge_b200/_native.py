"""Loader for the native sm_100a library (``_lib/libnfb200.so``).

The library has a C ABI and is loaded with ctypes; every entry point takes raw
device pointers, sizes, strides and a ``cudaStream_t`` and returns a
``cudaError_t``. :func:`call` checks that code and raises.

``HAS_NATIVE`` is the capability flag (the counterpart of the reference's
``HAS_TRITON``, nuvla_forge/kernels/utils.py:7-20): True when a CUDA device is
visible and the library loaded. On a machine with a GPU a missing or broken
library is an error, not a silent fallback, unless ``NFB_ALLOW_REFERENCE=1``
is set; ``NUVLA_FORGE_DISABLE_NATIVE=1`` forces the pure-PyTorch reference.
``NFB_DEBUG=1`` loads the debug build (device bounds checks that report through
:func:`debug_status` instead of faulting).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_int64, c_uint32, c_uint64, c_void_p

import torch

from ._build import build, lib_path

P = c_void_p
I = c_int
L = c_int64
F = c_float
U32 = c_uint32
U64 = c_uint64

DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_SIGS: dict[str, tuple] = {
    "nfb_num_sms": (I, []),
    "nfb_norm_fwd": (I, [I, I, I, P, P, P, P, P, P, P, P, P, L, L, L, L, L, L, L, L, L, L, F, I, P]),
    "nfb_norm_bwd_P": (L, [L, L, L]),
    "nfb_norm_set_status": (None, [P]),
    "nfb_norm_set_impl": (None, [I]),
    "nfb_norm_get_impl": (I, []),
    "nfb_norm_bwd": (I, [I, I, I, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P,
                         L, L, L, L, L, L, L, L, L, L, L, L, I, P]),
    "nfb_swiglu_fwd": (I, [I, P, P, P, L, L, L, L, L, P]),
    "nfb_swiglu_bwd": (I, [I, P, P, P, P, P, L, L, L, L, L, L, L, P]),
    "nfb_image_normalize": (I, [I, P, P, L, L, P, P, P]),
    "nfb_image_patchify": (I, [I, P, P, L, I, I, I, I, P, P, P]),
    "nfb_adamw_flat": (I, [P, P, P, P, P, L, F, F, F, F, F, L, F, P, F, P]),
    "nfb_sumsq_slots": (I, []),
    "nfb_sumsq": (I, [I, P, L, F, P, P, P, I, P]),
    "nfb_accum": (I, [I, P, P, L, F, I, P]),
    "nfb_cast": (I, [I, I, P, P, L, F, P]),
    "nfb_comm_flag_bytes": (I, []),
    "nfb_ar_twoshot": (I, [P, I, I, P, P, L, L, L, L, I, F, U32, U64, P, I, P]),
    "nfb_ar_oneshot": (I, [P, I, I, P, P, L, L, L, L, I, F, U32, U64, P, I, P]),
    "nfb_ar_pipelined": (I, [P, I, I, P, P, L, L, L, L, I, I, F, U32, U64, P, L, I, P]),
    "nfb_rs_push": (I, [P, I, I, P, L, L, L, I, F, U32, U64, P, P, I, I, P]),
    "nfb_rs_push_sumsq": (I, [P, I, I, P, L, L, L, I, F, U32, U64, P, P, I, P, P, P, I, P]),
    "nfb_rs_f32": (I, [P, I, I, L, L, L, I, F, U32, U64, P, P, P, P, P, I, I, I, P]),
    "nfb_rs_adamw": (I, [P, I, I, L, L, L, I, F, U32, U64, P, P, P, P, L, F, F, F, F, F, L, F, I, I, P]),
    "nfb_allgather": (I, [P, I, I, L, L, P, L, I, U32, U64, P, I, P]),
    "nfb_allreduce_scalar": (I, [P, I, I, L, P, L, I, U32, U64, P, P]),
    "nfb_wait_flag": (I, [P, U32, U64, P, P]),
    "nfb_ce_rows": (I, [I, P, L, P, L, L, L, P, P, P]),
    "nfb_count_valid": (I, [P, L, L, P, P]),
    "nfb_tc_gemm_bf16": (I, [P, P, P, I, I, I, L, L, L, I, P, P]),
    "nfb_tc_gemm_ex": (I, [P, P, P, I, I, I, L, L, L, I, I, I, I, P, P]),
    "nfb_attn_fwd": (I, [P, P, P, P, P, I, I, I, I, I, I, L, L, L, L, L, L, L, L, L, L, L, L, I, F, P, P]),
    "nfb_attn_bwd_scratch_bytes": (L, [I, I, I, I]),
    "nfb_attn_fwd_trace": (None, [P]),
    "nfb_mma_rate": (I, [I, I, I, P, I, P]),
    "nfb_attn_bwd_trace": (None, [P]),
    "nfb_attn_bwd": (I, [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, P, I, F, P, P]),
    "nfb_ce_tc_tiles": (I, [I]),
    "nfb_ce_tc_stats": (I, [P, L, P, L, P, I, I, I, P, P, P, P, P]),
    "nfb_ce_tc_merge": (I, [P, P, P, P, P, I, I, L, P, P, P]),
    "nfb_ce_tc_grad": (I, [P, L, P, L, P, P, P, L, I, I, I, P, L, P, P]),
    "nfb_ag_gemm": (I, [P, I, I, L, L, P, L, L, L, I, I, P, L, I, P, L, P, P, P]),
    "nfb_ag_gemm_max_nblocks": (I, []),
    "nfb_copy_async": (I, [P, P, L, P]),
    "nfb_gemm": (I, [P, P, P, I, I, I, L, L, L, I, I, I, P, P, L, P, P]),
    "nfb_gemm_acc": (I, [P, P, P, I, I, I, L, L, L, I, I, I, I, P, L, U32, P, P]),
    "nfb_gemm_acc_splits": (I, [I, I, I]),
    "nfb_gemm_max_clusters": (I, []),
    "nfb_gemm_small": (I, [I, I, P, L, L, P, L, L, P, L, L, P, I, I, I, I, P]),
    "nfb_gemm_last_error": (ctypes.c_char_p, []),
    "nfb_debug_status": (U32, []),
    "nfb_debug_reset": (None, []),
    "nfb_is_debug_build": (I, []),
    "nfb_gemm_swiglu_fwd": (I, [P, P, P, P, I, I, I, L, L, L, L, P, P]),
    "nfb_gemm_swiglu_bwd": (I, [P, P, P, P, I, I, I, L, L, L, L, P, P]),
}

_lib = None
_load_error: str | None = None


def _want_native() -> bool:
    return os.environ.get("NUVLA_FORGE_DISABLE_NATIVE", "0") != "1"


DEBUG = os.environ.get("NFB_DEBUG", "0") == "1"


def _load():
    global _lib, _load_error
    if _lib is not None or _load_error is not None:
        return _lib
    path = lib_path(DEBUG)
    try:
        if not path.exists() and os.environ.get("NFB_NO_AUTOBUILD", "0") != "1":
            build(debug=DEBUG)
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    except Exception as exc:  # noqa: BLE001 - reported through HAS_NATIVE / require()
        _load_error = f"{type(exc).__name__}: {exc}"
    return _lib


def cuda_ok() -> bool:
    return torch.cuda.is_available()


def _compute_has_native() -> bool:
    if not _want_native() or not cuda_ok():
        return False
    lib = _load()
    if lib is None:
        if os.environ.get("NFB_ALLOW_REFERENCE", "0") == "1":
            return False
        raise RuntimeError(
            "CUDA is available but the native library failed to load "
            f"({_load_error}). Build it with `python -m nuvla_forge_b200._build` "
            "or set NFB_ALLOW_REFERENCE=1 to run the slow PyTorch reference."
        )
    return True


HAS_NATIVE: bool = _compute_has_native()


def lib():
    """The loaded CDLL (loads it on first use; raises if unavailable)."""
    l = _load()
    if l is None:
        raise RuntimeError(f"native library unavailable: {_load_error}")
    return l


class NativeError(RuntimeError):
    pass


_launches = [0]


def reset_launch_count() -> None:
    _launches[0] = 0


def launch_count() -> int:
    """Number of native kernel launches issued through :func:`call` since the last reset."""
    return _launches[0]


_fns: dict[str, object] = {}


def call(name: str, *args) -> int:
    """Call ``name`` (one kernel launch) and raise if it returns a non-zero CUDA error code."""
    fn = _fns.get(name)
    if fn is None:
        fn = _fns[name] = getattr(lib(), name)
    _launches[0] += 1
    rc = fn(*args)
    if rc != 0:
        detail = ""
        if name.startswith("nfb_gemm"):
            detail = f": {lib().nfb_gemm_last_error().decode()}"
        raise NativeError(f"{name} failed with CUDA error {rc} ({_err_name(rc)}){detail}")
    return rc


_ERR_NAMES = {1: "cudaErrorInvalidValue", 2: "cudaErrorMemoryAllocation", 98: "cudaErrorInvalidDeviceFunction",
              209: "cudaErrorNoKernelImageForDevice", 700: "cudaErrorIllegalAddress",
              701: "cudaErrorLaunchOutOfResources", 715: "cudaErrorIllegalInstruction",
              716: "cudaErrorMisalignedAddress", 719: "cudaErrorLaunchFailure"}


def _err_name(rc: int) -> str:
    return _ERR_NAMES.get(rc, "see cuda_runtime_api.h")


# Pointers and streams are passed as plain ints (None for NULL): every entry point declares
# c_void_p argument types, so ctypes converts them without a wrapper object per argument.
def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream(device: torch.device | None = None) -> int:
    """The current CUDA stream of ``device`` (default: the current device) as a ``cudaStream_t`` value."""
    if _raw_stream is not None and (device is None or isinstance(device, torch.device)):
        idx = device.index if device is not None else None
        return _raw_stream(torch.cuda.current_device() if idx is None else idx)
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt not in DT:
        raise TypeError(f"unsupported dtype {dt}")
    return DT[dt]


def num_sms() -> int:
    return int(lib().nfb_num_sms())


def loaded_library_path() -> str | None:
    return str(lib_path(DEBUG)) if _lib is not None else None


def debug_status() -> int:
    """First failed device check of the debug build ((4 << 24) | site), 0 if none (always 0 in release)."""
    return int(lib().nfb_debug_status())


def debug_reset() -> None:
    lib().nfb_debug_reset()

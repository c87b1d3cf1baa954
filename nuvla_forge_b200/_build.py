"""Build the native library ``nuvla_forge_b200/_lib/libnfb200.so``.

All CUDA sources under ``csrc/`` are compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with plain ``nvcc``, in parallel,
into position-independent objects that are linked into one shared library with
a C ABI. No torch headers are involved, so a full rebuild takes seconds and the
library can be loaded by any process (Python through ctypes, or C/C++).

    python -m nuvla_forge_b200._build            # incremental
    python -m nuvla_forge_b200._build --clean    # full rebuild
    python -m nuvla_forge_b200._build --debug    # libnfb200_debug.so: device bounds checks (-DNFB_DEBUG)

The debug library reports a failed device-side check (an out-of-range label, a
bad stride, ...) in a status word read by ``nfb_debug_status()`` instead of
faulting; ``NFB_DEBUG=1`` makes ``nuvla_forge_b200._native`` load it.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "_lib"
OBJDIR = LIBDIR / "obj"
LIBNAME = "libnfb200.so"
DEBUG_LIBNAME = "libnfb200_debug.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-warn-spills",
]


def nvcc_path() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin/ on PATH")


def lib_path(debug: bool = False) -> Path:
    return LIBDIR / (DEBUG_LIBNAME if debug else LIBNAME)


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, nvcc: str, extra: list[str], objdir: Path = OBJDIR) -> tuple[Path, str]:
    obj = objdir / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj, ""
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc, "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
               "-Xcompiler", "-pthread", *extra, "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(clean: bool = False, verbose: bool = False, extra: list[str] | None = None, debug: bool = False) -> Path:
    """Compile every source for sm_100a and link the shared library. Returns its path.

    ``debug`` builds ``libnfb200_debug.so`` (-DNFB_DEBUG, separate objects) instead.
    """
    extra = list(extra or [])
    objdir = OBJDIR
    if debug:
        extra.append("-DNFB_DEBUG")
        objdir = LIBDIR / "obj_debug"
    if clean and objdir.exists():
        shutil.rmtree(objdir)
    objdir.mkdir(parents=True, exist_ok=True)
    nvcc = nvcc_path()
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 4))) as ex:
        results = list(ex.map(lambda s: _compile(s, nvcc, extra, objdir), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for o, log in results:
            if log.strip():
                print(f"--- {o.name}\n{log}")
    out = lib_path(debug)
    newest = max(o.stat().st_mtime for o in objs)
    if clean or not out.exists() or out.stat().st_mtime < newest:
        tmp = out.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, out)
    return out


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--debug", action="store_true", help="build libnfb200_debug.so (device bounds checks)")
    args = ap.parse_args(argv)
    path = build(clean=args.clean, verbose=args.verbose, debug=args.debug)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Symmetric device memory for the fused NVLink collectives (CUDA IPC peer mappings).

Every rank allocates one buffer of the same size (native ``nfb_ipc_alloc``),
exports a CUDA IPC handle, gathers all ranks' handles through the process
group, and maps every peer's buffer into its own address space. The native
kernels (csrc/comm.cu) receive all ranks' base pointers and address peers with
plain loads and stores over NVLink. No NVLink multicast object is created.

Layout (byte offsets): [flags | scalar exchange | data ...]. ``alloc`` hands
out 256-byte-aligned regions of the data area (every rank must reserve the
same sequence).

Each collective kind uses its own flag *slot*; every launch takes the next
epoch of its slot (a host counter that all ranks advance identically, because
all ranks launch the same collectives in the same order). Bounded waits in the
kernels report into ``status``; :meth:`check` raises ``CommTimeout``.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from .. import _native as nat

SLOT_DDP, SLOT_RS, SLOT_AG, SLOT_SCALAR, SLOT_TEST, SLOT_DDP_SMALL, SLOT_DDP_B = 0, 1, 2, 3, 4, 5, 6


class CommTimeout(RuntimeError):
    """A fused collective gave up waiting for a peer (the peer died or stalled)."""


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def decode_status(v: int) -> str:
    code, where = (v >> 24) & 0xFF, v & 0xFFFFFF
    kinds = {1: "barrier timeout", 2: "flag timeout", 3: "bad argument"}
    return f"{kinds.get(code, f'code {code}')} at site {where & 0xFFFF} (peer {where >> 16})"


def _ipc_fns():
    lib = nat.lib()
    for name, res, args in (("nfb_ipc_handle_bytes", ctypes.c_int, []),
                            ("nfb_ipc_alloc", ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p),
                                                             ctypes.c_void_p]),
                            ("nfb_ipc_open", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
                            ("nfb_ipc_close", ctypes.c_int, [ctypes.c_void_p]),
                            ("nfb_ipc_free", ctypes.c_int, [ctypes.c_void_p]),
                            ("nfb_device_synchronize", ctypes.c_int, [])):
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class SymmetricWorkspace:
    def __init__(self, data_bytes: int, group: dist.ProcessGroup | None = None,
                 device: torch.device | None = None, timeout_s: float | None = None):
        self.group = group or dist.group.WORLD
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        lib = _ipc_fns()
        self._lib = lib
        self.flag_off = 0
        self.scalar_off = _align(int(lib.nfb_comm_flag_bytes()))
        self.data_off = self.scalar_off + 256
        self.total = self.data_off + _align(max(int(data_bytes), 256))
        hb = int(lib.nfb_ipc_handle_bytes())
        handle = (ctypes.c_char * hb)()
        local = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            rc = lib.nfb_ipc_alloc(self.total, ctypes.byref(local), ctypes.cast(handle, ctypes.c_void_p))
            if rc != 0:
                raise RuntimeError(f"nfb_ipc_alloc({self.total}) failed with CUDA error {rc}")
            lib.nfb_device_synchronize()
        self._local = local.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        ptrs, self._opened = [], []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._local)
                    continue
                p = ctypes.c_void_p()
                buf = (ctypes.c_char * hb).from_buffer_copy(h)
                rc = lib.nfb_ipc_open(ctypes.cast(buf, ctypes.c_void_p), ctypes.byref(p))
                if rc != 0:
                    raise RuntimeError(f"rank {self.rank}: opening rank {r}'s IPC handle failed (CUDA error {rc})")
                ptrs.append(p.value)
                self._opened.append(p.value)
        self.bases = (ctypes.c_uint64 * self.world)(*ptrs)
        self._cursor = self.data_off
        self.epochs = [0] * 8
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        t = timeout_s if timeout_s is not None else float(os.environ.get("NFB_COMM_TIMEOUT_S", "30"))
        self.timeout_ns = int(t * 1e9)
        dist.barrier(self.group)

    def alloc(self, nbytes: int) -> int:
        """Reserve ``nbytes`` of the data area; returns the region's byte offset."""
        off = self._cursor
        end = off + _align(nbytes)
        if end > self.total:
            raise MemoryError(f"symmetric workspace exhausted ({end} > {self.total} bytes)")
        self._cursor = end
        return off

    def local_ptr(self, off: int = 0) -> int:
        return self._local + off

    def next_epoch(self, slot: int) -> int:
        self.epochs[slot] = (self.epochs[slot] + 1) & 0x7FFFFFFF
        return self.epochs[slot]

    def bases_ptr(self) -> ctypes.c_void_p:
        return ctypes.cast(self.bases, ctypes.c_void_p)

    def check(self) -> None:
        v = int(self.status.item())
        if v:
            raise CommTimeout(f"rank {self.rank}: fused collective failed: {decode_status(v)}")

    def close(self) -> None:
        """Unmap peers and free the local buffer (call on every rank, with no kernel in flight)."""
        if getattr(self, "_local", None) is None:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self._opened:
                self._lib.nfb_ipc_close(ctypes.c_void_p(p))
            self._lib.nfb_ipc_free(ctypes.c_void_p(self._local))
        self._opened = []
        self._local = None


def symmetric_memory_available() -> bool:
    if not (torch.cuda.is_available() and nat.HAS_NATIVE and dist.is_initialized()):
        return False
    if os.environ.get("NFB_DISABLE_FUSED_COMM", "0") == "1":
        return False
    return dist.get_world_size() <= 8

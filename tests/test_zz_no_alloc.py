"""The allocation-free norm backward (nfb_norm_bwd_noalloc) against the regular entry point.

nfb_norm_bwd_noalloc is for callers that cannot allocate device memory when
they run the backward (a host framework with a fixed memory plan, or plugin
code whose contract forbids allocating); it keeps its scratch in a file-scope
device array instead of taking scratch buffers. This file is named so pytest
collects it last. It calls the exported C symbol through ctypes and compares
every output with nfb_norm_bwd's on two calls in a row, using the same
tolerance as the other kernel tests, and checks that oversized problems are
rejected with a clear message.
"""

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL_BF16 = 1.2e-2


def _lib():
    from nuvla_forge_b200 import _native as nat

    assert nat.HAS_NATIVE, "native library must load on a GPU box"
    lib = ctypes.CDLL(str(nat.lib_path()))
    fn = lib.nfb_norm_bwd_noalloc
    fn.restype = c_int
    fn.argtypes = [c_int, c_int, c_int] + [c_void_p] * 14 + [c_int64] * 11 + [c_int, c_void_p]
    err = lib.nfb_noalloc_last_error
    err.restype = ctypes.c_char_p
    err.argtypes = []
    return nat, fn, err


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _problem(B, T, N, seed):
    from nuvla_forge_b200.ops.norm import GATE_VEC, _fwd

    g = torch.Generator(device=DEV).manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g, device=DEV).to(torch.bfloat16)  # noqa: E731
    x, y = mk(B * T, N), mk(B * T, N)
    cond = mk(B, 3 * N) * 0.5
    gate, scale, shift = cond[:, :N], cond[:, N:2 * N], cond[:, 2 * N:]
    w = (1 + 0.1 * mk(N)).to(torch.bfloat16)
    h, _, rstd, w, wf = _fwd(x, y, gate, w, scale, shift, T, 1e-6, GATE_VEC, True)
    dh_up, dout = mk(B * T, N), mk(B * T, N)
    return dict(x=x, y=y, gate=gate, w=w, scale=scale, h=h, rstd=rstd, dh_up=dh_up, dout=dout, wf=wf)


def _outputs(B, T, N):
    mk = lambda *s: torch.empty(*s, device=DEV, dtype=torch.bfloat16)  # noqa: E731
    return dict(dx=mk(B * T, N), dy=mk(B * T, N), dgate=mk(B, N), dscale=mk(B, N), dshift=mk(B, N), dweight=mk(N))


def _args_common(nat, p, o):
    return [p["dh_up"], p["dout"], p["h"], p["y"], p["gate"], p["w"], p["scale"], p["rstd"],
            o["dx"], o["dy"], o["dgate"], o["dscale"], o["dshift"], o["dweight"]]


def _run_regular(nat, p, B, T, N):
    from nuvla_forge_b200.ops.norm import GATE_VEC

    o = _outputs(B, T, N)
    M = B * T
    P = int(nat.lib().nfb_norm_bwd_P(M, N, B))
    partials = torch.empty(B * P * 3 * N, device=DEV)
    dwb = torch.empty(B * N, device=DEV)
    tickets = torch.zeros(B + 1, dtype=torch.int32, device=DEV)
    nat.call("nfb_norm_bwd", 1, GATE_VEC, 1, *[nat.ptr(t) for t in _args_common(nat, p, o)],
             nat.ptr(partials), nat.ptr(dwb), nat.ptr(tickets), M, N, T, P,
             N, N, N, N, N, N, p["gate"].stride(0), p["scale"].stride(0), p["wf"], nat.stream())
    return o


def _run_noalloc(nat, fn, p, B, T, N):
    from nuvla_forge_b200.ops.norm import GATE_VEC

    o = _outputs(B, T, N)
    rc = fn(1, GATE_VEC, 1, *[t.data_ptr() for t in _args_common(nat, p, o)], B * T, N, T,
            N, N, N, N, N, N, p["gate"].stride(0), p["scale"].stride(0), p["wf"],
            torch.cuda.current_stream().cuda_stream)
    return rc, o


@pytest.mark.parametrize("B,T,N", [(4, 96, 1024), (8, 2048, 1536), (2, 7, 768)])
def test_noalloc_matches_regular_entry_point_twice(B, T, N):
    nat, fn, err = _lib()
    p = _problem(B, T, N, seed=B * 131 + N)
    ref = _run_regular(nat, p, B, T, N)
    for _ in range(2):   # two calls in a row share (and must re-initialise) the scratch
        rc, out = _run_noalloc(nat, fn, p, B, T, N)
        assert rc == 0, err().decode()
        torch.cuda.synchronize()
        for k in ref:
            assert _rel(out[k], ref[k]) < TOL_BF16, (k, _rel(out[k], ref[k]))


def test_noalloc_rejects_oversized_problem():
    nat, fn, err = _lib()
    B, T, N = 200, 1, 8192          # needs 200*8192*4 floats > 4 MiB of scratch
    dummy = torch.zeros(1, device=DEV)
    ptrs = [dummy.data_ptr()] * 14
    rc = fn(1, 2, 1, *ptrs, B * T, N, T, N, N, N, N, N, N, N, N, 0, torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert "too large" in err().decode()

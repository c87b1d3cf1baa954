"""The debug build (-DNFB_DEBUG): device-side checks report a bad label instead of reading past a row."""

import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_debug_checks_compile_for_sm100a(tmp_path):
    """The checked translation units cross-compile with the debug macro (no GPU needed)."""
    from nuvla_forge_b200._build import ARCH_FLAGS, CSRC, NVCC_FLAGS, nvcc_path

    for src in ("ce_rows.cu", "ipc.cu"):
        r = subprocess.run([nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-DNFB_DEBUG", "-I", str(CSRC), "-c",
                            str(CSRC / src), "-o", str(tmp_path / (src + ".o"))], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


_CHILD = textwrap.dedent("""
    import torch
    from nuvla_forge_b200 import _native as nat
    assert nat.lib().nfb_is_debug_build() == 1
    nat.debug_reset()
    V = 1000
    logits = torch.randn(4, V, device="cuda").to(torch.bfloat16)
    targets = torch.tensor([3, V + 7, -100, 5], device="cuda")         # row 1: label out of range
    count = torch.tensor([3.0], device="cuda")
    loss = torch.zeros(4, device="cuda")
    nat.call("nfb_ce_rows", 1, nat.ptr(logits), V, nat.ptr(targets), 4, V, -100, nat.ptr(count), nat.ptr(loss),
             nat.stream())
    torch.cuda.synchronize()                                            # the context is still healthy
    print("STATUS", hex(nat.debug_status()), float(loss[0]), float(loss[3]))
""")


@pytest.mark.gpu
def test_out_of_range_label_is_reported_not_read():
    env = dict(os.environ, NFB_DEBUG="1", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", _CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("STATUS")][0].split()
    assert int(line[1], 16) == (4 << 24) | 1001, line
    assert float(line[2]) > 0 and float(line[3]) > 0                   # the valid rows were processed

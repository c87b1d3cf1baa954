"""The reference's import path and CLI (``nuvla_forge``) run on this implementation."""

import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_imports_resolve_to_native_ops():
    from nuvla_forge.kernels import HAS_TRITON, chunked_cross_entropy, fused_adaln_residual_rmsnorm, fused_swiglu
    from nuvla_forge.kernels.reference import swiglu_ref
    from nuvla_forge.model import NuVLA, NuVLAConfig
    from nuvla_forge.profiling import StepTimer, roofline_note

    import nuvla_forge_b200.ops as ops

    assert fused_swiglu is ops.fused_swiglu and chunked_cross_entropy is ops.chunked_cross_entropy
    assert fused_adaln_residual_rmsnorm is ops.fused_adaln_residual_rmsnorm
    assert isinstance(HAS_TRITON, bool)
    a, b = torch.randn(4, 16), torch.randn(4, 16)
    assert torch.allclose(fused_swiglu(a, b, force_reference=True), swiglu_ref(a, b))
    assert NuVLA(NuVLAConfig(vision_depth=1, fusion_depth=1, text_depth=1, dit_depth=1)) is not None
    assert callable(StepTimer) and isinstance(roofline_note(100.0, 1000.0), str)


def test_reference_cli_entry_point():
    r = subprocess.run([sys.executable, "-m", "nuvla_forge.train", "--help"], cwd=ROOT, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "--preset" in r.stdout and "--fused-kernels" in r.stdout


def test_reference_arm_is_not_shadowed_by_the_alias():
    """bench.py --impl reference must import the unmodified reference from baseline/_ref, not this alias."""
    ref = os.path.join(ROOT, "baseline", "_ref", "nuvla_forge")
    if not os.path.isdir(ref):
        pytest.skip("reference not installed in baseline/_ref")
    code = ("import sys; sys.path.insert(0, 'baseline'); from ref_arm import _import_reference; "
            "m, err = _import_reference(); print(err or m.__file__)")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and os.path.join("baseline", "_ref", "nuvla_forge") in r.stdout, r.stdout + r.stderr

"""The FMA-pipe 2^x used by the attention softmax (csrc/tc_gemm.cuh:ex2_poly), emulated step by step
in fp32 with NumPy from the constants in the source, against 2^x in float64."""

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "nuvla_forge_b200" / "csrc" / "tc_gemm.cuh"


def _coeffs():
    text = SRC.read_text()
    return [np.float32(float(re.search(rf"kExp2C{i} = ([0-9.e+-]+)f;", text).group(1))) for i in range(4)]


def ex2_poly(x):
    c0, c1, c2, c3 = _coeffs()
    x = np.maximum(np.asarray(x, dtype=np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic)).astype(np.float32)
    p = ((c3 * f + c2) * f + c1) * f + c0
    p = p.astype(np.float32)
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_below_bf16_resolution():
    x = np.linspace(-120.0, 8.0, 2_000_001, dtype=np.float32)
    got = ex2_poly(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 1e-4, rel.max()        # bf16 resolution is 2^-8 = 3.9e-3


def test_underflow_and_masked_inputs_give_tiny_nonnegative_values():
    got = ex2_poly(np.array([-np.inf, -1e30, -200.0, -126.0, -125.5], dtype=np.float32))
    assert np.all(np.isfinite(got)) and np.all(got >= 0.0) and np.all(got < 2.0 ** -124)


def test_integer_inputs_are_exact_powers_up_to_the_polynomial_constant():
    x = np.arange(-100, 9, dtype=np.float32)
    got = ex2_poly(x).astype(np.float64)
    assert np.allclose(got, np.exp2(x.astype(np.float64)) * float(_coeffs()[0]), rtol=1e-7)

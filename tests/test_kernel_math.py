"""Finite-difference checks (float64 NumPy) of the backward formulas the native kernels implement.

Parity: reference tests/test_kernel_math.py (adaLN backward vs central
differences, zero-gate identity, SwiGLU, CE with ignored rows and the
valid-count denominator). The formulas here are transcriptions of what
csrc/norm.cu, csrc/swiglu.cu and csrc/ce_rows.cu compute, including the
shared-accumulator identities the one-launch norm backward relies on
(dscale[b] = w * A_b, dweight = sum_b (1 + scale[b]) * A_b).
"""

import numpy as np

EPS = 1e-6
H = 1e-6
RTOL = 1e-6


def fwd(x, y, gate, w, scale, shift, T):
    g = np.repeat(gate, T, 0)
    s = np.repeat(scale, T, 0)
    sh = np.repeat(shift, T, 0)
    h = x + g * y
    rstd = 1.0 / np.sqrt((h * h).mean(-1, keepdims=True) + EPS)
    out = h * rstd * w * (1 + s) + sh
    return h, out


def bwd(x, y, gate, w, scale, shift, T, dh_up, dout):
    """The kernel's backward, written with its per-sample accumulators."""
    M, N = x.shape
    B = M // T
    g = np.repeat(gate, T, 0)
    s = np.repeat(scale, T, 0)
    h = x + g * y
    rstd = 1.0 / np.sqrt((h * h).mean(-1, keepdims=True) + EPS)
    xhat = h * rstd
    ws = w * (1 + s)
    dxh = dout * ws
    dot = (dxh * xhat).sum(-1, keepdims=True) / N
    dh = dh_up + rstd * (dxh - xhat * dot)
    dx = dh
    dy = dh * g
    A = (dout * xhat).reshape(B, T, N).sum(1)
    D = dout.reshape(B, T, N).sum(1)
    G = (dh * y).reshape(B, T, N).sum(1)
    dscale = w * A
    dweight = ((1 + scale) * A).sum(0)
    return dx, dy, G, dweight, dscale, D


def _fd(fn, arr, idx):
    old = arr[idx]
    arr[idx] = old + H
    fp = fn()
    arr[idx] = old - H
    fm = fn()
    arr[idx] = old
    return (fp - fm) / (2 * H)


def test_adaln_backward_matches_finite_differences():
    rng = np.random.default_rng(0)
    B, T, N = 2, 3, 8
    x, y = rng.standard_normal((B * T, N)), rng.standard_normal((B * T, N))
    gate, scale, shift = (rng.standard_normal((B, N)) for _ in range(3))
    w = 1 + 0.1 * rng.standard_normal(N)
    dh_up, dout = rng.standard_normal((B * T, N)), rng.standard_normal((B * T, N))
    args = [x, y, gate, w, scale, shift]

    def loss():
        h, out = fwd(*args, T)
        return (h * dh_up).sum() + (out * dout).sum()

    grads = bwd(*args, T, dh_up, dout)
    for arr, g in zip(args, grads):
        for idx in np.ndindex(arr.shape):
            num = _fd(loss, arr, idx)
            assert abs(num - g[idx]) <= RTOL * max(1.0, abs(num)) + 1e-7, (idx, num, g[idx])


def test_zero_gate_is_identity_on_residual():
    rng = np.random.default_rng(1)
    x, y = rng.standard_normal((6, 16)), rng.standard_normal((6, 16))
    z = np.zeros((2, 16))
    h, _ = fwd(x, y, z, np.ones(16), z, z, 3)
    assert np.array_equal(h, x)


def test_swiglu_backward():
    rng = np.random.default_rng(2)
    a, b, d = (rng.standard_normal(50) for _ in range(3))
    sig = 1 / (1 + np.exp(-a))
    da = d * b * sig * (1 + a * (1 - sig))
    db = d * a * sig

    def loss():
        s = 1 / (1 + np.exp(-a))
        return (a * s * b * d).sum()

    for arr, g in ((a, da), (b, db)):
        for i in range(arr.size):
            num = _fd(loss, arr, (i,))
            assert abs(num - g[i]) <= RTOL * max(1.0, abs(num)) + 1e-7


def _ce(hid, W, tgt, ignore=-100):
    logits = hid @ W.T
    valid = tgt != ignore
    n = max(valid.sum(), 1)
    m = logits.max(-1, keepdims=True)
    lse = (m + np.log(np.exp(logits - m).sum(-1, keepdims=True)))[:, 0]
    loss = np.where(valid, lse - logits[np.arange(len(tgt)), np.where(valid, tgt, 0)], 0.0).sum() / n
    p = np.exp(logits - lse[:, None])
    p[np.arange(len(tgt)), np.where(valid, tgt, 0)] -= 1
    p = p * valid[:, None] / n
    return loss, p @ W, p.T @ hid


def test_ce_gradients_with_ignored_rows():
    rng = np.random.default_rng(3)
    hid, W = rng.standard_normal((7, 5)), rng.standard_normal((11, 5)) * 0.5
    tgt = rng.integers(0, 11, 7)
    tgt[[1, 4]] = -100
    loss, dh, dW = _ce(hid, W, tgt)
    for arr, g in ((hid, dh), (W, dW)):
        for idx in np.ndindex(arr.shape):
            num = _fd(lambda: _ce(hid, W, tgt)[0], arr, idx)
            assert abs(num - g[idx]) <= RTOL * max(1.0, abs(num)) + 1e-7
    assert np.all(dh[[1, 4]] == 0)


def test_ce_mean_uses_valid_count():
    rng = np.random.default_rng(4)
    hid, W = rng.standard_normal((6, 4)), rng.standard_normal((9, 4))
    tgt = rng.integers(0, 9, 6)
    full, _, _ = _ce(hid, W, tgt)
    tgt2 = tgt.copy()
    tgt2[:3] = -100
    part, _, _ = _ce(hid, W, tgt2)
    per_row = []
    for i in range(3, 6):
        l, _, _ = _ce(hid[i:i + 1], W, tgt[i:i + 1])
        per_row.append(l)
    assert abs(part - np.mean(per_row)) < 1e-12
    assert abs(full - part) > 1e-6

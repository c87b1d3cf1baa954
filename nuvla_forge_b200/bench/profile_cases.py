"""Small, self-contained launches of each native kernel, for profiling one kernel at a time.

    python -m nuvla_forge_b200.bench.profile_cases --case norm_bwd [--iters 3]
    ncu --set full --clock-control none -k regex:norm_bwd -s 1 -c 1 -o prof \\
        python -m nuvla_forge_b200.bench.profile_cases --case norm_bwd

Every case keeps its working set above the 126 MB L2 (so DRAM counters mean
something) and below ~2 GB on the device, and launches its kernel ``--iters``
times (the first launch is a warm-up to skip with ``-s``).
"""

from __future__ import annotations

import argparse

import torch

CASES = {}


def case(fn):
    CASES[fn.__name__] = fn
    return fn


def _bf(*s, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*s, generator=g, device="cuda").to(torch.bfloat16)


@case
def norm_fwd(iters):
    """adaLN seam forward at BASELINE config 2: x, y [8*2048, 1536] bf16."""
    from ..ops import fused_adaln_residual_rmsnorm
    b, t, n = 8, 2048, 1536
    x, y, cond, w = _bf(b * t, n), _bf(b * t, n, seed=1), _bf(b, 3 * n, seed=2), _bf(n, seed=3)
    with torch.no_grad():
        for _ in range(iters):
            fused_adaln_residual_rmsnorm(x, y, cond[:, :n], w, cond[:, n:2 * n], cond[:, 2 * n:], t)


@case
def norm_bwd(iters):
    """adaLN seam backward at BASELINE config 2 (one launch incl. per-sample reductions)."""
    from ..ops import fused_adaln_residual_rmsnorm
    b, t, n = 8, 2048, 1536
    leaves = [v.requires_grad_(True) for v in (_bf(b * t, n), _bf(b * t, n, seed=1), _bf(b, n, seed=2),
                                                _bf(n, seed=3), _bf(b, n, seed=4), _bf(b, n, seed=5))]
    dh, do = _bf(b * t, n, seed=6), _bf(b * t, n, seed=7)
    h, o = fused_adaln_residual_rmsnorm(*leaves, tokens_per_sample=t)
    for _ in range(iters):
        torch.autograd.backward([h, o], [dh, do], retain_graph=True)


@case
def add_rmsnorm_bwd(iters):
    """Residual add + RMSNorm backward at the ViT shape of the 1b config (the training step's norm seam)."""
    from ..ops import add_rmsnorm
    x = _bf(98304, 1024).requires_grad_(True)
    y = _bf(98304, 1024, seed=1).requires_grad_(True)
    w = _bf(1024, seed=2).requires_grad_(True)
    h, o = add_rmsnorm(x, y, w)
    dh, do = _bf(98304, 1024, seed=3), _bf(98304, 1024, seed=4)
    for _ in range(iters):
        torch.autograd.grad([h, o], [x, y, w], [dh, do], retain_graph=True)


@case
def rmsnorm_bwd(iters):
    """Plain RMSNorm backward at the ViT shape of the 1b config: [98304, 1024]."""
    from ..ops import rmsnorm
    x = _bf(98304, 1024).requires_grad_(True)
    w = _bf(1024, seed=1).requires_grad_(True)
    out = rmsnorm(x, w)
    d = _bf(98304, 1024, seed=2)
    for _ in range(iters):
        out.backward(d, retain_graph=True)


@case
def swiglu_fwd(iters):
    """SwiGLU forward at BASELINE config 2: a, b [16384, 4096]."""
    from ..ops import fused_swiglu
    a, b = _bf(16384, 4096), _bf(16384, 4096, seed=1)
    with torch.no_grad():
        for _ in range(iters):
            fused_swiglu(a, b)


@case
def swiglu_bwd(iters):
    """SwiGLU backward at BASELINE config 2."""
    from ..ops import fused_swiglu
    a, b = _bf(16384, 4096).requires_grad_(True), _bf(16384, 4096, seed=1).requires_grad_(True)
    out = fused_swiglu(a, b)
    d = _bf(16384, 4096, seed=2)
    for _ in range(iters):
        out.backward(d, retain_graph=True)


@case
def tc_gemm(iters):
    """tcgen05 GEMM core, 8192 x 8192 x 8192 bf16 -> bf16."""
    from ..ops.ce_tc import tc_gemm as g
    a, b = _bf(8192, 8192), _bf(8192, 8192, seed=1)
    for _ in range(iters):
        g(a, b)


@case
def gemm_pair(iters):
    """CTA-pair tcgen05 GEMM, 8192 x 8192 x 8192 bf16 -> bf16 (forward layout)."""
    from ..ops.linear import gemm
    a, b = _bf(8192, 8192), _bf(8192, 8192, seed=1)
    for _ in range(iters):
        gemm(a, b)


@case
def gemm_pair_vit_qkv(iters):
    """CTA-pair GEMM at the ViT qkv forward shape (K = 1024), 32768 tokens: y [32768, 3072]."""
    from ..ops.linear import gemm
    x, w = _bf(32768, 1024), _bf(3072, 1024, seed=1)
    for _ in range(iters):
        gemm(x, w)


@case
def gemm_pair_swiglu_bwd(iters):
    """Down projection's input gradient with the SwiGLU backward in its epilogue, ViT MLP shape at 24
    images: dY [24576, 1024], W_down [1024, 4096], ab / d_ab [24576, 8192] (interleaved gate / up)."""
    from .. import _native as nat
    from ..ops import linear as L
    M, F, D = 24576, 4096, 1024
    dy, wd = _bf(M, D), _bf(D, F, seed=1)
    ab = _bf(M, 2 * F, seed=2)
    dab = torch.empty_like(ab)
    st = L.status_word(dy.device)
    for _ in range(iters):
        nat.call("nfb_gemm_swiglu_bwd", nat.ptr(dy), nat.ptr(wd), nat.ptr(ab), nat.ptr(dab), M, F, D, dy.stride(0),
                 wd.stride(0), ab.stride(0), dab.stride(0), nat.ptr(st), nat.stream(dy.device))
    torch.cuda.synchronize()
    L.check_status()


@case
def gemm_pair_wgrad(iters):
    """CTA-pair GEMM weight gradient at the backbone proj shape: dW [2048, 2048] fp32 over 27136 tokens."""
    from ..ops.linear import gemm_acc
    dy, x = _bf(27136, 2048), _bf(27136, 2048, seed=1)
    dw = torch.zeros(2048, 2048, dtype=torch.float32, device="cuda")
    for _ in range(iters):
        gemm_acc(dy, x, dw, a_mn=True, b_mn=True)


@case
def attn_bwd(iters):
    """Native attention backward at the ViT shape, 24 images: q, k, v, o, do [24, 1024, 16, 64] bf16."""
    from ..ops import flash_attn
    B, S, H, D = 24, 1024, 16, 64
    qkv = _bf(B, S, 3 * H, D)
    q, k, v = qkv.split([H, H, H], dim=2)
    out, lse = flash_attn.attention_fwd(q, k, v)
    dout = _bf(B, S, H, D, seed=1)
    for _ in range(iters):
        flash_attn.attention_bwd(q, k, v, out, dout, lse)


@case
def ce_tc(iters):
    """Cross entropy on tcgen05 at BASELINE config 2: hidden [16384, 2048], W [32000, 2048]."""
    from ..ops.ce_tc import cross_entropy_tc
    h = _bf(16384, 2048).requires_grad_(True)
    w = (_bf(32000, 2048, seed=1) * 0.02).requires_grad_(True)
    t = torch.randint(0, 32000, (16384,), device="cuda")
    for _ in range(iters):
        cross_entropy_tc(h, w, t).backward()


@case
def adamw(iters):
    """Flat AdamW over 256M parameters (fp32 master, grads, moments + bf16 copy)."""
    from .. import _native as nat
    n = 256 * 2**20
    p, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    v.abs_()
    lp = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    for i in range(iters):
        nat.call("nfb_adamw_flat", nat.ptr(p), nat.ptr(g), nat.ptr(m), nat.ptr(v), nat.ptr(lp), n, 3e-4, 0.9, 0.999,
                 1e-8, 0.01, i + 1, 1.0, nat.ptr(None), 0.0, nat.stream())


@case
def patchify(iters):
    """uint8 -> normalised bf16 patch rows for 96 images of 448x448 (one micro-batch of the 1b config)."""
    from ..ops import patchify_images
    img = torch.randint(0, 256, (96, 448, 448, 3), dtype=torch.uint8, device="cuda")
    for _ in range(iters):
        patchify_images(img, 14)


@case
def ag_gemm(iters):
    """All-gather-fused GEMM on one GPU (world 1: the gather copies the local shard):
    a 64 MB parameter unit, first GEMM M=4096, N=5120, K=3072 (the 3b qkv shape)."""
    import ctypes

    from .. import _native as nat
    numel = 32 * 2**20
    prefix, M, N, K = 8192, 4096, 5120, 3072
    shard = _bf(numel)
    full = torch.empty(numel, dtype=torch.bfloat16, device="cuda")
    x = _bf(M, K, seed=1)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ready = torch.zeros(1024, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    bases = (ctypes.c_uint64 * 1)(shard.data_ptr())
    for _ in range(iters):
        nat.call("nfb_ag_gemm", ctypes.cast(bases, ctypes.c_void_p), 0, 1, 0, numel * 2, nat.ptr(full), prefix * 2,
                 numel * 2, prefix * 2, N, K, nat.ptr(x), K, M, nat.ptr(y), N, nat.ptr(ready), nat.ptr(status),
                 nat.stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0, hex(int(status.item()))


@case
def attn_fwd(iters):
    """tcgen05 attention forward, ViT shape (24 images x 1024 patches, 16 heads, D 64; ~600 MB of q/k/v/o)."""
    from ..ops import flash_attn
    q = _bf(24, 1024, 16, 64)
    kv = _bf(24, 1024, 32, 64, seed=1)
    k, v = kv.split([16, 16], dim=2)
    for _ in range(iters):
        flash_attn.attention_fwd(q, k, v, False)
    torch.cuda.synchronize()
    flash_attn.check_status()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True, choices=sorted(CASES))
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args(argv)
    CASES[args.case](args.iters)
    torch.cuda.synchronize()
    print(f"{args.case}: ok")


if __name__ == "__main__":
    main()

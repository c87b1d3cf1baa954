"""Native sm_100a kernels against fp32 PyTorch references (parity: reference tests/test_kernels.py)."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _nat():
    from nuvla_forge_b200 import _native as nat

    assert nat.HAS_NATIVE, "native library must load on a GPU box"
    return nat


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


TOL = {torch.float32: 2e-5, torch.bfloat16: 1.2e-2, torch.float16: 2e-3}


def _gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def _inputs(b, t, n, dtype, seed=0, strided=True):
    g = _gen(seed)
    mk = lambda *s: torch.randn(*s, generator=g, device=DEV, dtype=torch.float32).to(dtype)  # noqa: E731
    x, y = mk(b * t, n), mk(b * t, n)
    cond = mk(b, 6 * n) * 0.5
    if strided:  # gate/scale/shift as row-strided views of one [B, 6N] tensor (the model's layout)
        gate, scale, shift = cond[:, :n], cond[:, 2 * n: 3 * n], cond[:, 4 * n: 5 * n]
    else:
        gate, scale, shift = cond[:, :n].contiguous(), cond[:, n: 2 * n].contiguous(), cond[:, 2 * n: 3 * n].contiguous()
    w = (1 + 0.1 * mk(n)).to(dtype)
    return x, y, gate, w, scale, shift


SHAPES = [(2, 16, 256), (4, 32, 1024), (3, 7, 768), (1, 64, 1536), (2, 5, 1000), (8, 128, 2048),
          (2, 300, 4096), (1, 37, 8192)]


@pytest.fixture(params=[0, 1], ids=["warp_team", "pipelined"])
def norm_impl(request):
    """Run a norm test with the warp/team kernels (0, default) and the bulk-copy pipelined kernels (1)."""
    _nat()
    from nuvla_forge_b200.ops import norm

    norm.set_impl(request.param)
    yield request.param
    norm.check_status()
    norm.set_impl(0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
def test_adaln_fwd_bwd(shape, dtype, norm_impl):
    _nat()
    from nuvla_forge_b200.ops import fused_adaln_residual_rmsnorm
    from nuvla_forge_b200.ops.reference import adaln_residual_rmsnorm_ref

    b, t, n = shape
    base = _inputs(b, t, n, dtype)
    leaves_n = [v.detach().clone().requires_grad_(True) for v in base]
    leaves_r = [v.detach().clone().float().requires_grad_(True) for v in base]
    h, o = fused_adaln_residual_rmsnorm(*leaves_n, tokens_per_sample=t)
    hr, orf = adaln_residual_rmsnorm_ref(*leaves_r, tokens_per_sample=t)
    g = _gen(1)
    dh = torch.randn(h.shape, generator=g, device=DEV).to(dtype)
    do = torch.randn(o.shape, generator=g, device=DEV).to(dtype)
    tol = TOL[dtype]
    assert rel_err(h, hr) < tol and rel_err(o, orf) < tol
    (h.float() * dh.float() + o.float() * do.float()).sum().backward()
    (hr * dh.float() + orf * do.float()).sum().backward()
    for name, a, r in zip(["x", "y", "gate", "weight", "scale", "shift"], leaves_n, leaves_r):
        assert a.grad is not None, name
        assert rel_err(a.grad, r.grad) < 2 * tol, (name, rel_err(a.grad, r.grad))


def test_adaln_deterministic():
    _nat()
    from nuvla_forge_b200.ops import fused_adaln_residual_rmsnorm

    outs = []
    for _ in range(2):
        leaves = [v.detach().clone().requires_grad_(True) for v in _inputs(8, 256, 1536, torch.bfloat16)]
        h, o = fused_adaln_residual_rmsnorm(*leaves, tokens_per_sample=256)
        (h.float().sum() + (o.float() ** 2).sum()).backward()
        outs.append([l.grad.clone() for l in leaves])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rmsnorm_variants(dtype, norm_impl):
    _nat()
    from nuvla_forge_b200.ops import add_rmsnorm, rmsnorm
    from nuvla_forge_b200.ops.reference import add_rmsnorm_ref, rmsnorm_ref

    x, y, gate, w, scale, shift = _inputs(4, 33, 512, dtype)
    xs = [x.clone().requires_grad_(True), x.float().clone().requires_grad_(True)]
    ws = [w.clone().requires_grad_(True), w.float().clone().requires_grad_(True)]
    out = rmsnorm(xs[0], ws[0])
    ref = rmsnorm_ref(xs[1], ws[1])
    assert rel_err(out, ref) < TOL[dtype]
    (out.float() ** 2).sum().backward()
    (ref ** 2).sum().backward()
    assert rel_err(xs[0].grad, xs[1].grad) < 2 * TOL[dtype]
    assert rel_err(ws[0].grad, ws[1].grad) < 2 * TOL[dtype]
    # modulated
    sc = [scale.clone().requires_grad_(True), scale.float().clone().requires_grad_(True)]
    sh = [shift.clone().requires_grad_(True), shift.float().clone().requires_grad_(True)]
    out = rmsnorm(x, w, scale=sc[0], shift=sh[0], tokens_per_sample=33)
    T = 33
    ref = rmsnorm_ref(x.float(), w.float()) * (1 + sc[1].repeat_interleave(T, 0)) + sh[1].repeat_interleave(T, 0)
    assert rel_err(out, ref) < TOL[dtype]
    out.float().sum().backward()
    ref.sum().backward()
    assert rel_err(sc[0].grad, sc[1].grad) < 2 * TOL[dtype]
    assert rel_err(sh[0].grad, sh[1].grad) < 2 * TOL[dtype]
    # residual add + norm
    h, o = add_rmsnorm(x, y, w)
    hr, orf = add_rmsnorm_ref(x.float(), y.float(), w.float())
    assert rel_err(h, hr) < TOL[dtype] and rel_err(o, orf) < TOL[dtype]


def test_norm_impls_agree():
    """Pipelined and warp/team kernels give the same result up to fp32 summation order."""
    _nat()
    from nuvla_forge_b200.ops import fused_adaln_residual_rmsnorm, norm

    base = _inputs(8, 256, 1536, torch.bfloat16)
    res = []
    for impl in (1, 0):
        norm.set_impl(impl)
        leaves = [v.detach().clone().requires_grad_(True) for v in base]
        h, o = fused_adaln_residual_rmsnorm(*leaves, tokens_per_sample=256)
        (h.float().sum() + (o.float() ** 2).sum()).backward()
        res.append([h, o] + [l.grad for l in leaves])
    norm.set_impl(0)
    norm.check_status()
    for a, b in zip(*res):
        assert rel_err(a, b) < 1e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(64, 512), (128, 2048), (17, 333), (4096, 1536)])
def test_swiglu(shape, dtype):
    _nat()
    from nuvla_forge_b200.ops import fused_swiglu
    from nuvla_forge_b200.ops.reference import swiglu_ref

    g = _gen(3)
    a0 = torch.randn(*shape, generator=g, device=DEV).to(dtype)
    b0 = torch.randn(*shape, generator=g, device=DEV).to(dtype)
    a, b = a0.clone().requires_grad_(True), b0.clone().requires_grad_(True)
    ar, br = a0.float().clone().requires_grad_(True), b0.float().clone().requires_grad_(True)
    out = fused_swiglu(a, b)
    ref = swiglu_ref(ar, br)
    assert rel_err(out, ref) < TOL[dtype]
    d = torch.randn(*shape, generator=g, device=DEV)
    out.backward(d.to(dtype))
    ref.backward(d)
    assert rel_err(a.grad, ar.grad) < 2 * TOL[dtype]
    assert rel_err(b.grad, br.grad) < 2 * TOL[dtype]


def test_swiglu_packed():
    _nat()
    from nuvla_forge_b200.ops import swiglu_packed
    from nuvla_forge_b200.ops.reference import swiglu_ref

    g = _gen(4)
    ab0 = torch.randn(3, 50, 2 * 704, generator=g, device=DEV).to(torch.bfloat16)
    ab = ab0.clone().requires_grad_(True)
    abr = ab0.float().clone().requires_grad_(True)
    out = swiglu_packed(ab)
    ref = swiglu_ref(abr[..., :704], abr[..., 704:])
    assert rel_err(out, ref) < TOL[torch.bfloat16]
    d = torch.randn(out.shape, generator=g, device=DEV)
    out.backward(d.to(torch.bfloat16))
    ref.backward(d)
    assert rel_err(ab.grad, abr.grad) < 2 * TOL[torch.bfloat16]


def test_image_kernels():
    _nat()
    from nuvla_forge_b200.ops import normalise_images, patchify_images
    from nuvla_forge_b200.ops.reference import normalise_images_ref, patchify_ref

    g = torch.Generator().manual_seed(0)
    chw = torch.randint(0, 256, (2, 6, 3, 32, 48), dtype=torch.uint8, generator=g).to(DEV)
    for dt in (torch.bfloat16, torch.float32):
        assert rel_err(normalise_images(chw, dt), normalise_images_ref(chw, dt)) < TOL[dt]
    hwc = torch.randint(0, 256, (5, 448, 448, 3), dtype=torch.uint8, generator=g).to(DEV)
    out = patchify_images(hwc, 14)
    ref = patchify_ref(hwc, 14, 592)
    assert out.shape == (5, 1024, 592)
    assert rel_err(out, ref) < TOL[torch.bfloat16]
    assert torch.count_nonzero(out[..., 588:]) == 0
    hwc2 = torch.randint(0, 256, (3, 128, 128, 3), dtype=torch.uint8, generator=g).to(DEV)
    assert rel_err(patchify_images(hwc2, 16), patchify_ref(hwc2, 16, 768)) < TOL[torch.bfloat16]
    # 24 patches per strip: one full staging group of 16 and a partial one
    hwc3 = torch.randint(0, 256, (2, 28, 336, 3), dtype=torch.uint8, generator=g).to(DEV)
    out3 = patchify_images(hwc3, 14)
    assert rel_err(out3, patchify_ref(hwc3, 14, 592)) < TOL[torch.bfloat16]
    assert torch.count_nonzero(out3[..., 588:]) == 0


@pytest.mark.parametrize("m,h,v,chunk", [(256, 128, 1000, 64), (1000, 384, 32000, 1024), (96, 64, 4096, 4096)])
def test_chunked_ce(m, h, v, chunk):
    _nat()
    from nuvla_forge_b200.ops import chunked_cross_entropy
    from nuvla_forge_b200.ops.reference import chunked_cross_entropy_ref

    g = _gen(5)
    hid0 = torch.randn(m, h, generator=g, device=DEV).to(torch.bfloat16)
    w0 = (torch.randn(v, h, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    tgt = torch.randint(0, v, (m,), generator=g, device=DEV)
    tgt[::7] = -100
    hid, w = hid0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
    hr, wr = hid0.float().clone().requires_grad_(True), w0.float().clone().requires_grad_(True)
    loss = chunked_cross_entropy(hid, w, tgt, chunk_size=chunk)
    ref = chunked_cross_entropy_ref(hr, wr, tgt)
    assert abs(float(loss) - float(ref)) < 2e-3 * max(1.0, abs(float(ref)))
    loss.backward()
    ref.backward()
    assert rel_err(hid.grad, hr.grad) < 2e-2
    assert rel_err(w.grad, wr.grad) < 2e-2
    assert torch.count_nonzero(hid.grad[::7]) == 0


def test_chunked_ce_all_ignored():
    _nat()
    from nuvla_forge_b200.ops import chunked_cross_entropy

    hid = torch.randn(32, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(500, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    tgt = torch.full((32,), -100, device=DEV)
    loss = chunked_cross_entropy(hid, w, tgt)
    loss.backward()
    assert torch.isfinite(loss) and float(loss) == 0.0
    assert torch.count_nonzero(hid.grad) == 0


def test_chunked_ce_peak_memory_below_naive():
    """The logits never exist as an [M, V] fp32 tensor: the native CE's peak allocation during
    forward + backward stays below half the naive CE's and below one fp32 logits tensor."""
    _nat()
    from nuvla_forge_b200.ops import chunked_cross_entropy
    from nuvla_forge_b200.ops.reference import chunked_cross_entropy_ref

    m, h, v = 4096, 384, 32000
    g = _gen(11)
    hid = torch.randn(m, h, generator=g, device=DEV).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(v, h, generator=g, device=DEV) * 0.05).to(torch.bfloat16).requires_grad_(True)
    tgt = torch.randint(0, v, (m,), generator=g, device=DEV)

    def peak(fn):
        hid.grad = w.grad = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        fn().backward()
        torch.cuda.synchronize()
        return torch.cuda.max_memory_allocated() - base

    native = peak(lambda: chunked_cross_entropy(hid, w, tgt, chunk_size=1024))
    naive = peak(lambda: chunked_cross_entropy_ref(hid, w, tgt))
    assert native < naive / 2, (native, naive)
    assert native < 0.75 * m * v * 4, native


def test_flat_adamw_matches_torch():
    _nat()
    from nuvla_forge_b200.optim.adamw import FlatAdamW

    class Space:
        pass

    n = 10_003
    g = _gen(6)
    p0 = torch.randn(n, generator=g, device=DEV)
    sp = Space()
    sp.master = p0.clone()
    sp.grads = torch.zeros(n, device=DEV)
    sp.params = torch.zeros(n, device=DEV, dtype=torch.bfloat16)
    opt = FlatAdamW(sp, lr=1e-2, weight_decay=0.05, max_grad_norm=1.0)
    ref_p = torch.nn.Parameter(p0.clone())
    ref = torch.optim.AdamW([ref_p], lr=1e-2, weight_decay=0.05, fused=False, foreach=False)
    for _ in range(4):
        grad = torch.randn(n, generator=g, device=DEV) * 3
        sp.grads.copy_(grad)
        opt.step()
        ref_p.grad = grad.clone()
        torch.nn.utils.clip_grad_norm_([ref_p], 1.0)
        ref.step()
        assert abs(float(opt.grad_norm()) - float(grad.norm())) < 1e-3 * float(grad.norm())
    assert rel_err(sp.master, ref_p.detach()) < 1e-5
    assert rel_err(sp.params, ref_p.detach()) < 5e-3


def test_sumsq_and_accum():
    nat = _nat()
    g = _gen(7)
    x = torch.randn(1_000_001, generator=g, device=DEV)
    parts = torch.empty(int(nat.lib().nfb_sumsq_slots()), device=DEV)
    ticket = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.zeros(1, device=DEV)
    for _ in range(2):
        nat.call("nfb_sumsq", 0, nat.ptr(x), x.numel(), 1.0, nat.ptr(parts), nat.ptr(ticket), nat.ptr(out), 0,
                 nat.stream())
        assert abs(float(out) - float(x.double().square().sum())) < 1e-3 * float(x.double().square().sum())
    assert int(ticket) == 0
    dst = torch.randn(4099, generator=g, device=DEV)
    src = torch.randn(4099, generator=g, device=DEV).to(torch.bfloat16)
    exp = dst + src.float()
    nat.call("nfb_accum", 1, nat.ptr(dst), nat.ptr(src), 4099, 1.0, 0, nat.stream())
    assert rel_err(dst, exp) < 1e-6
    nat.call("nfb_accum", 1, nat.ptr(dst), nat.ptr(src), 4099, 1.0, 1, nat.stream())
    assert rel_err(dst, src.float()) < 1e-6


def test_bounded_wait_times_out_and_context_survives():
    """A wait on a flag nothing sets gives up after its limit and reports a status; the GPU stays usable."""
    nat = _nat()
    import time

    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    t0 = time.time()
    nat.call("nfb_wait_flag", nat.ptr(flag), 1, int(0.2e9), nat.ptr(status), nat.stream())
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(status) != 0 and (int(status) >> 24) == 2
    assert dt < 5.0
    x = torch.ones(1024, device=DEV)
    assert float(x.sum()) == 1024.0


def test_allreduce_kernel_single_rank():
    """The fused all-reduce on a 1-rank 'group' (peer table = own buffer): out = bf16(in) * scale."""
    nat = _nat()
    n = 8 * 4096 + 8 * 17
    flag_bytes = int(nat.lib().nfb_comm_flag_bytes())
    buf = torch.zeros(flag_bytes + 2 * n * 2 + 4096, dtype=torch.uint8, device=DEV)
    base = buf.data_ptr()
    bases = (ctypes.c_uint64 * 1)(base)
    src = torch.randn(n, device=DEV)
    dst = torch.empty(n, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    send_off = (flag_bytes + 255) // 256 * 256
    recv_off = send_off + (n * 2 + 255) // 256 * 256
    for epoch in (1, 2):
        nat.call("nfb_ar_twoshot", ctypes.cast(bases, ctypes.c_void_p), 0, 1, nat.ptr(src), nat.ptr(dst), n,
                 send_off, recv_off, 0, 0, 0.5, epoch, int(1e9), nat.ptr(status), 8, nat.stream())
        torch.cuda.synchronize()
        assert int(status) == 0
        exp = src.to(torch.bfloat16).float() * 0.5
        assert rel_err(dst, exp.to(torch.bfloat16).float()) < 1e-6

"""The CTA-pair tcgen05 GEMM (forward, input gradient, weight gradient) against fp32 references."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _rand(g, *shape):
    return torch.randn(*shape, generator=g, device=DEV).to(torch.bfloat16)


SHAPES = [(128, 256, 64), (256, 256, 64), (300, 1000, 200), (129, 264, 72), (8, 3072, 1024),
          (1000, 512, 8), (2048, 2048, 1024), (4096, 3072, 1024)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_forward_matches_fp32(M, N, K, out_dtype):
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(M + 7 * N + K)
    a, b = _rand(g, M, K), _rand(g, N, K)
    c = L.gemm(a, b, out_dtype=out_dtype)
    torch.cuda.synchronize()
    L.check_status()
    ref = a.float() @ b.float().t()
    assert rel_err(c, ref) < (1e-5 if out_dtype == torch.float32 else 5e-3), rel_err(c, ref)


@pytest.mark.parametrize("M,N,K", [(300, 1000, 200), (1024, 512, 256), (64, 264, 96)])
def test_forward_bias_residual(M, N, K):
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(11)
    a, b = _rand(g, M, K), _rand(g, N, K)
    bias, res = _rand(g, N), _rand(g, M, N)
    c = L.gemm(a, b, bias=bias, residual=res)
    ref = a.float() @ b.float().t() + bias.float() + res.float()
    assert rel_err(c, ref) < 5e-3


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_input_grad_matches_fp32(M, N, K):
    """dx = dy W with W [N, K] read MN-major (GEMM K = N)."""
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(3 * M + N + K)
    dy, w = _rand(g, M, N), _rand(g, N, K)
    dx = L.input_grad(dy, w)
    torch.cuda.synchronize()
    L.check_status()
    assert rel_err(dx, dy.float() @ w.float()) < 5e-3


@pytest.mark.parametrize("M,N,K", SHAPES + [(16384, 1024, 1024), (27136, 512, 2048)])
def test_weight_grad_matches_fp32(M, N, K):
    """dW = dy^T x, both operands MN-major, fp32 output, split over M (the token dimension)."""
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(5 * M + N + K)
    dy, x = _rand(g, M, N), _rand(g, M, K)
    c = torch.empty(N, K, dtype=torch.float32, device=DEV)
    L.gemm_acc(dy, x, c, a_mn=True, b_mn=True)
    torch.cuda.synchronize()
    L.check_status()
    ref = dy.float().t() @ x.float()
    assert rel_err(c, ref) < 1e-5, rel_err(c, ref)


@pytest.mark.parametrize("splits", [1, 2, 3, 7])
def test_weight_grad_splits_accumulate_deterministic(splits):
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(17)
    M, N, K = 8192, 768, 512
    dy, x = _rand(g, M, N), _rand(g, M, K)
    base = torch.randn(N, K, generator=g, device=DEV)
    c1 = base.clone()
    L.gemm_acc(dy, x, c1, a_mn=True, b_mn=True, accumulate=True, splits=splits)
    c2 = base.clone()
    L.gemm_acc(dy, x, c2, a_mn=True, b_mn=True, accumulate=True, splits=splits)
    torch.cuda.synchronize()
    L.check_status()
    ref = base + dy.float().t() @ x.float()
    assert rel_err(c1, ref) < 1e-5
    assert torch.equal(c1, c2)   # fixed summation order: bit-identical


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_operand_layouts_and_strides(a_mn, b_mn):
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(23)
    M, N, K = 520, 392, 136
    a, b = _rand(g, M, K), _rand(g, N, K)
    big_a = torch.zeros((K, M + 24) if a_mn else (M, K + 24), dtype=torch.bfloat16, device=DEV)
    big_b = torch.zeros((K, N + 40) if b_mn else (N, K + 40), dtype=torch.bfloat16, device=DEV)
    if a_mn:
        big_a[:, 8:8 + M] = a.t()
        a_in = big_a[:, 8:8 + M]
    else:
        big_a[:, 16:16 + K] = a
        a_in = big_a[:, 16:16 + K]
    if b_mn:
        big_b[:, 0:N] = b.t()
        b_in = big_b[:, 0:N]
    else:
        big_b[:, 8:8 + K] = b
        b_in = big_b[:, 8:8 + K]
    c = L.gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out_dtype=torch.float32)
    assert rel_err(c, a.float() @ b.float().t()) < 1e-5


@pytest.mark.parametrize("shape", [(4, 96, 256, 512), (2, 333, 1024, 264)])
@pytest.mark.parametrize("bias", [False, True])
def test_linear_autograd_matches_fp32(shape, bias):
    from nuvla_forge_b200.ops import linear as L

    B, T, K, N = shape
    g = torch.Generator(device=DEV).manual_seed(B * T + K)
    x = _rand(g, B, T, K).requires_grad_(True)
    w = (_rand(g, N, K) * 0.05).requires_grad_(True)
    b = _rand(g, N).requires_grad_(True) if bias else None
    r = _rand(g, B, T, N).requires_grad_(True)
    y = L.linear(x, w, b, residual=r)
    dy = _rand(g, B, T, N)
    y.backward(dy)
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    bf = b.detach().float().requires_grad_(True) if bias else None
    rf = r.detach().float().requires_grad_(True)
    yf = torch.nn.functional.linear(xf, wf, bf) + rf
    yf.backward(dy.float())
    assert rel_err(y, yf) < 5e-3
    assert rel_err(x.grad, xf.grad) < 5e-3
    assert rel_err(w.grad, wf.grad) < 5e-3
    assert rel_err(r.grad, rf.grad) < 1e-6
    if bias:
        assert rel_err(b.grad, bf.grad) < 5e-3


class _Owner:
    """A gradient owner as the DDP runtime registers one: fp32 buffer, overwrite then accumulate."""

    def __init__(self, w):
        self.buf = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        self.fresh = True
        self.done = 0

    def grad_target(self, w):
        ow = self.fresh
        self.fresh = False
        return self.buf, ow

    def grad_done(self, w):
        self.done += 1


@pytest.mark.parametrize("K,N", [(512, 256), (3, 1024), (1024, 3)])
def test_linear_owner_receives_fp32_grad(K, N):
    """With a registered owner the weight gradient lands in its fp32 buffer (overwrite, then +=)."""
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(K + N)
    w = torch.nn.Parameter(_rand(g, N, K) * 0.1)
    owner = _Owner(w)
    w._nfb_grad_owner = owner
    x1, x2 = _rand(g, 300, K), _rand(g, 300, K)
    d1, d2 = _rand(g, 300, N), _rand(g, 300, N)
    L.linear(x1, w).backward(d1)
    L.linear(x2, w).backward(d2)
    torch.cuda.synchronize()
    assert w.grad is None and owner.done == 2
    ref = d1.float().t() @ x1.float() + d2.float().t() @ x2.float()
    assert rel_err(owner.buf, ref) < 1e-5


@pytest.mark.parametrize("K,N", [(3, 1024), (1024, 3), (256, 48)])
def test_small_linear_autograd(K, N):
    """Widths the tensor-core tiles cannot cover run the CUDA-core kernel in all three products."""
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(K * N)
    x = _rand(g, 128, K).requires_grad_(True)
    w = _rand(g, N, K).requires_grad_(True)
    b = _rand(g, N).requires_grad_(True)
    y = L.linear(x, w, b)
    dy = _rand(g, 128, N)
    y.backward(dy)
    xf, wf, bf = (t.detach().float().requires_grad_(True) for t in (x, w, b))
    torch.nn.functional.linear(xf, wf, bf).backward(dy.float())
    assert rel_err(x.grad, xf.grad) < 5e-3
    assert rel_err(w.grad, wf.grad) < 5e-3
    assert rel_err(b.grad, bf.grad) < 5e-3


@pytest.mark.parametrize("M,D,F", [(300, 256, 384), (1024, 512, 1024), (4096, 1024, 4096), (130, 2048, 5632)])
@pytest.mark.parametrize("residual", [False, True])
def test_fused_swiglu_mlp_matches_fp32(M, D, F, residual):
    """Gate/up GEMM with SwiGLU in its epilogue, down projection, and the fused backward, against fp32."""
    from nuvla_forge_b200.ops import linear as L

    g = torch.Generator(device=DEV).manual_seed(M + D + F)
    x = (_rand(g, M, D)).requires_grad_(True)
    wg, wu = _rand(g, F, D) * 0.05, _rand(g, F, D) * 0.05
    wd = (_rand(g, D, F) * 0.05).requires_grad_(True)
    w_gu = L.interleave_gate_up(wg, wu).contiguous().requires_grad_(True)
    r = _rand(g, M, D).requires_grad_(True) if residual else None
    y = L.swiglu_mlp(x, w_gu, wd, r)
    dy = _rand(g, M, D)
    y.backward(dy)
    torch.cuda.synchronize()
    L.check_status()
    xf = x.detach().float().requires_grad_(True)
    wgf, wuf = wg.float().requires_grad_(True), wu.float().requires_grad_(True)
    wdf = wd.detach().float().requires_grad_(True)
    a, b = xf @ wgf.t(), xf @ wuf.t()
    yf = (torch.nn.functional.silu(a) * b) @ wdf.t()
    if residual:
        rf = r.detach().float().requires_grad_(True)
        yf = yf + rf
    yf.backward(dy.float())
    assert rel_err(y, yf) < 1e-2
    assert rel_err(x.grad, xf.grad) < 1e-2
    assert rel_err(wd.grad, wdf.grad) < 1e-2
    gg, gu = L.split_gate_up_rows(w_gu.grad)
    assert rel_err(gg, wgf.grad) < 1e-2 and rel_err(gu, wuf.grad) < 1e-2
    if residual:
        assert rel_err(r.grad, rf.grad) < 1e-6


def test_swiglu_mlp_module_state_dict_keeps_reference_layout():
    """The interleaved weight is split back into w_gate / w_up on save and re-interleaved on load."""
    from nuvla_forge_b200.models.layers import SwiGLUMLP

    m = SwiGLUMLP(256, 512).cuda().to(torch.bfloat16)
    sd = m.state_dict()
    assert set(sd) == {"w_gate.weight", "w_up.weight", "w_down.weight"}
    m2 = SwiGLUMLP(256, 512).cuda().to(torch.bfloat16)
    m2.load_state_dict(sd)
    assert torch.equal(m2.w_gate_up, m.w_gate_up)
    x = _rand(torch.Generator(device=DEV).manual_seed(1), 64, 256)
    ref = (torch.nn.functional.silu(x.float() @ sd["w_gate.weight"].float().t())
           * (x.float() @ sd["w_up.weight"].float().t())) @ sd["w_down.weight"].float().t()
    assert rel_err(m(x), ref) < 1e-2

"""The tcgen05/TMEM GEMM core and the tcgen05 cross entropy against fp32 references."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 1000, 200), (129, 257, 72), (1024, 2048, 2048),
                                   (4096, 4096, 1024)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_tc_gemm_matches_fp32(M, N, K, out_dtype):
    from nuvla_forge_b200.ops import ce_tc

    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    b = torch.randn(N, K, generator=g, device=DEV).to(torch.bfloat16)
    c = ce_tc.tc_gemm(a, b, out_dtype)
    torch.cuda.synchronize()
    ce_tc.check_status()
    ref = a.float() @ b.float().t()
    assert rel_err(c, ref) < (1e-5 if out_dtype == torch.float32 else 5e-3), rel_err(c, ref)


def test_tc_gemm_strided_operands():
    from nuvla_forge_b200.ops import ce_tc

    g = torch.Generator(device=DEV).manual_seed(9)
    big_a = torch.randn(256, 512, generator=g, device=DEV).to(torch.bfloat16)
    big_b = torch.randn(384, 320, generator=g, device=DEV).to(torch.bfloat16)
    a, b = big_a[:, 64:192], big_b[:, 8:136]      # row strides 512 / 320, K = 128
    c = ce_tc.tc_gemm(a, b, torch.float32)
    assert rel_err(c, a.float() @ b.float().t()) < 1e-5


@pytest.mark.parametrize("a_mn,b_mn", [(True, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (304, 1000, 200), (136, 264, 72), (2048, 2048, 1024)])
def test_tc_gemm_mn_major_operands(M, N, K, a_mn, b_mn):
    """Operands stored transposed ([K, M] / [K, N], MN contiguous) against fp32, plus fp32 accumulate."""
    from nuvla_forge_b200.ops import ce_tc

    g = torch.Generator(device=DEV).manual_seed(3 * M + N + K)
    a = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    b = torch.randn(N, K, generator=g, device=DEV).to(torch.bfloat16)
    a_in = a.t().contiguous() if a_mn else a
    b_in = b.t().contiguous() if b_mn else b
    ref = a.float() @ b.float().t()
    c = ce_tc.tc_gemm(a_in, b_in, torch.float32, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    ce_tc.check_status()
    assert rel_err(c, ref) < 1e-5, rel_err(c, ref)
    base = torch.randn(M, N, generator=g, device=DEV)
    acc = base.clone()
    ce_tc.tc_gemm(a_in, b_in, a_mn=a_mn, b_mn=b_mn, out=acc, accumulate=True)
    assert rel_err(acc, base + ref) < 1e-5
    c16 = ce_tc.tc_gemm(a_in, b_in, torch.bfloat16, a_mn=a_mn, b_mn=b_mn)
    assert rel_err(c16, ref) < 5e-3


@pytest.mark.parametrize("M,H,V,chunk", [(256, 128, 1000, 128), (1000, 384, 32000, 512), (2048, 2048, 32000, 1024)])
def test_ce_tc_matches_reference(M, H, V, chunk):
    from nuvla_forge_b200.ops import ce_tc
    from nuvla_forge_b200.ops.reference import chunked_cross_entropy_ref

    g = torch.Generator(device=DEV).manual_seed(M + V)
    hid0 = torch.randn(M, H, generator=g, device=DEV).to(torch.bfloat16)
    w0 = (torch.randn(V, H, generator=g, device=DEV) * (1.0 / H ** 0.5)).to(torch.bfloat16)
    tgt = torch.randint(0, V, (M,), generator=g, device=DEV)
    tgt[::5] = -100
    hid, w = hid0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
    hr, wr = hid0.float().clone().requires_grad_(True), w0.float().clone().requires_grad_(True)
    loss = ce_tc.cross_entropy_tc(hid, w, tgt, chunk_rows=chunk)
    ref = chunked_cross_entropy_ref(hr, wr, tgt)
    loss.backward()
    ref.backward()
    torch.cuda.synchronize()
    ce_tc.check_status()
    assert abs(float(loss) - float(ref)) < 1e-3 * max(1.0, abs(float(ref))), (float(loss), float(ref))
    assert rel_err(hid.grad, hr.grad) < 2e-2
    assert rel_err(w.grad, wr.grad) < 2e-2
    assert torch.count_nonzero(hid.grad[::5]) == 0


def test_ce_dispatch_uses_tc_path():
    from nuvla_forge_b200 import _native as nat
    from nuvla_forge_b200.ops import chunked_cross_entropy

    hid = torch.randn(64, 256, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(512, 256, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    tgt = torch.randint(0, 512, (64,), device=DEV)
    nat.reset_launch_count()
    chunked_cross_entropy(hid, w, tgt).backward()
    assert nat.launch_count() >= 4   # count, stats, merge, grad


def test_mma_rate_probe_completes_and_reports_full_rate_for_n128():
    """nfb_mma_rate: back-to-back M128 N128 K16 MMAs run at (close to) the tensor core's full rate."""
    from nuvla_forge_b200 import _native as nat

    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    nat.call("nfb_mma_rate", 0, 128, 1024, nat.ptr(out), sms, nat.stream())
    torch.cuda.synchronize()
    cycles, ok = (int(v) for v in out.tolist())
    assert ok == 1
    assert 55 < cycles / 1024 < 90, cycles / 1024     # 64 cycles per instruction at the full rate

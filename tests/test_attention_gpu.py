"""The tcgen05 flash-attention forward (csrc/attention.cu) against an fp32 reference."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ref(q, k, v, causal, scale):
    B, Sq, Hq, D = q.shape
    Hk = k.shape[2]
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    kf = kf.repeat_interleave(Hq // Hk, dim=1)
    vf = vf.repeat_interleave(Hq // Hk, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        Sk = k.shape[1]
        qi = torch.arange(Sq, device=q.device)[:, None]
        ki = torch.arange(Sk, device=q.device)[None, :]
        s = s.masked_fill(ki > qi + (Sk - Sq), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(1, 2), lse


CASES = [  # B, Sq, Sk, Hq, Hkv, D, causal
    (2, 128, 128, 2, 2, 64, False),
    (1, 1024, 1024, 4, 4, 64, False),
    (2, 300, 300, 4, 2, 128, True),
    (1, 517, 517, 8, 2, 128, True),
    (2, 96, 1176, 6, 6, 64, False),
    (2, 16, 3392, 4, 4, 128, False),
    (1, 256, 200, 2, 1, 64, False),
    (1, 700, 700, 3, 3, 64, True),      # consecutive query tiles per CTA, unequal causal extents
    (2, 384, 384, 2, 2, 128, True),
]


@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv,D,causal", CASES)
def test_attention_fwd_matches_fp32(B, Sq, Sk, Hq, Hkv, D, causal):
    from nuvla_forge_b200.ops import flash_attn

    g = torch.Generator(device=DEV).manual_seed(Sq + Sk + D)
    # the projection-native layout: q, k, v are strided views of one fused [B, S, H + 2Hk, D] tensor when Sq == Sk
    if Sq == Sk:
        qkv = torch.randn(B, Sq, Hq + 2 * Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
        q, k, v = qkv.split([Hq, Hkv, Hkv], dim=2)
    else:
        q = torch.randn(B, Sq, Hq, D, generator=g, device=DEV).to(torch.bfloat16)
        kv = torch.randn(B, Sk, 2 * Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
        k, v = kv.split([Hkv, Hkv], dim=2)
    scale = D ** -0.5
    res = flash_attn.attention_fwd(q, k, v, causal, scale)
    assert res is not None
    out, lse = res
    torch.cuda.synchronize()
    flash_attn.check_status()
    ref_o, ref_lse = _ref(q, k, v, causal, scale)
    err = float((out.float() - ref_o).norm() / ref_o.norm())
    assert err < 1e-2, err
    assert torch.allclose(lse, ref_lse, atol=2e-2, rtol=1e-3), float((lse - ref_lse).abs().max())


def test_attention_native_autograd_path():
    """The opt-in op path: native forward, gradients via recompute, same as SDPA."""
    from nuvla_forge_b200.ops import attention, flash_attn

    g = torch.Generator(device=DEV).manual_seed(5)
    qkv = torch.randn(2, 256, 12, 64, generator=g, device=DEV).to(torch.bfloat16)
    a = qkv.clone().requires_grad_(True)
    b = qkv.clone().requires_grad_(True)
    flash_attn.enable(True)
    try:
        qa, ka, va = a.split([4, 4, 4], dim=2)
        oa = attention(qa, ka, va, causal=True)
    finally:
        flash_attn.enable(False)
    qb, kb, vb = b.split([4, 4, 4], dim=2)
    ob = attention(qb, kb, vb, causal=True)
    flash_attn.enable("auto")
    go = torch.randn_like(oa)
    oa.backward(go)
    ob.backward(go)
    assert float((oa.float() - ob.float()).norm() / ob.float().norm()) < 1e-2
    assert float((a.grad.float() - b.grad.float()).norm() / b.grad.float().norm()) < 2e-2


BWD_CASES = [  # B, Sq, Sk, Hq, Hkv, D, causal
    (2, 128, 128, 2, 2, 64, False),
    (1, 1024, 1024, 4, 4, 64, False),
    (2, 300, 300, 4, 2, 128, True),
    (1, 517, 517, 8, 2, 128, True),
    (2, 96, 1176, 6, 6, 64, False),
    (2, 16, 3392, 4, 4, 128, False),
    (1, 256, 200, 2, 1, 64, False),
    (1, 640, 640, 2, 2, 64, True),
]


@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv,D,causal", BWD_CASES)
def test_attention_bwd_matches_fp32(B, Sq, Sk, Hq, Hkv, D, causal):
    """Native dq / dk / dv against autograd through the fp32 reference (GQA, causal, cross lengths)."""
    from nuvla_forge_b200.ops import flash_attn

    g = torch.Generator(device=DEV).manual_seed(7 * Sq + Sk + D)
    q = torch.randn(B, Sq, Hq, D, generator=g, device=DEV).to(torch.bfloat16)
    kv = torch.randn(B, Sk, 2 * Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    k, v = kv.split([Hkv, Hkv], dim=2)
    scale = D ** -0.5
    out, lse = flash_attn.attention_fwd(q, k, v, causal, scale)
    dout = torch.randn(B, Sq, Hq, D, generator=g, device=DEV).to(torch.bfloat16)
    res = flash_attn.attention_bwd(q, k, v, out, dout, lse, causal, scale)
    assert res is not None
    dq, dk, dv = res
    torch.cuda.synchronize()
    flash_attn.check_status()
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref_o, _ = _ref(qf, kf, vf, causal, scale)
    ref_o.backward(dout.float())
    for name, got, want in (("dq", dq, qf.grad), ("dk", dk, kf.grad), ("dv", dv, vf.grad)):
        err = float((got.float() - want).norm() / want.norm())
        assert err < 2e-2, (name, err)


def test_attention_native_fwd_bwd_autograd_path():
    """The op path with both native kernels: gradients match SDPA's."""
    from nuvla_forge_b200.ops import attention, flash_attn

    g = torch.Generator(device=DEV).manual_seed(9)
    qkv = torch.randn(2, 384, 12, 128, generator=g, device=DEV).to(torch.bfloat16)
    a = qkv.clone().requires_grad_(True)
    b = qkv.clone().requires_grad_(True)
    flash_attn.enable(True)
    try:
        qa, ka, va = a.split([8, 2, 2], dim=2)
        oa = attention(qa, ka, va, causal=True)
        go = torch.randn_like(oa)
        oa.backward(go)
    finally:
        flash_attn.enable(False)
    qb, kb, vb = b.split([8, 2, 2], dim=2)
    ob = attention(qb, kb, vb, causal=True)
    ob.backward(go)
    flash_attn.enable("auto")
    assert float((oa.float() - ob.float()).norm() / ob.float().norm()) < 1e-2
    assert float((a.grad.float() - b.grad.float()).norm() / b.grad.float().norm()) < 2e-2


def test_auto_routing_uses_native_only_where_it_measured_faster():
    """Default routing: few queries into a long context go native, self-attention stays on SDPA."""
    from nuvla_forge_b200.ops import flash_attn

    g = torch.Generator(device=DEV).manual_seed(3)
    mk = lambda *s: torch.randn(*s, generator=g, device=DEV).to(torch.bfloat16)  # noqa: E731
    flash_attn.enable("auto")
    q, kv = mk(2, 16, 4, 64), mk(2, 3392, 8, 64)
    k, v = kv.split([4, 4], dim=2)
    assert flash_attn._native(q, k, v, False, None) is not None          # DiT cross-attention shape
    qs = mk(2, 1024, 12, 64)
    assert flash_attn._native(*qs.split([4, 4, 4], dim=2), False, None) is None   # self-attention
    flash_attn.enable(True)
    assert flash_attn._native(*qs.split([4, 4, 4], dim=2), False, None) is not None
    flash_attn.enable("auto")

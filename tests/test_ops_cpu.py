"""CPU checks of the op layer (reference paths, dispatch, API parity)."""

import pytest
import torch

from nuvla_forge_b200.kernels import (HAS_NATIVE, chunked_cross_entropy, fused_adaln_residual_rmsnorm,
                                      fused_swiglu)
from nuvla_forge_b200.kernels.reference import (adaln_residual_rmsnorm_ref, chunked_cross_entropy_ref,
                                                swiglu_ref)
from nuvla_forge_b200.ops import attention, patchify_images, rmsnorm
from nuvla_forge_b200.ops.reference import attention_ref, normalise_images_ref, patchify_ref


def test_capability_flag_off_on_cpu():
    assert HAS_NATIVE is False


def test_adaln_reference_manual_transcription():
    torch.manual_seed(0)
    B, T, N = 2, 3, 16
    x, y = torch.randn(B * T, N), torch.randn(B * T, N)
    gate, scale, shift, w = torch.randn(B, N), torch.randn(B, N), torch.randn(B, N), torch.randn(N)
    h, out = fused_adaln_residual_rmsnorm(x, y, gate, w, scale, shift, tokens_per_sample=T)
    g = gate.repeat_interleave(T, 0)
    hh = x + g * y
    ref = hh / torch.sqrt(hh.pow(2).mean(-1, keepdim=True) + 1e-6) * w * (1 + scale.repeat_interleave(T, 0)) \
        + shift.repeat_interleave(T, 0)
    assert torch.allclose(h, hh, atol=1e-6) and torch.allclose(out, ref, atol=1e-5)
    h2, o2 = adaln_residual_rmsnorm_ref(x, y, gate, w, scale, shift, T)
    assert torch.equal(h, h2) and torch.equal(out, o2)


def test_adaln_none_gate_and_modulation_defaults():
    x, y, w = torch.randn(6, 8), torch.randn(6, 8), torch.randn(8)
    h, out = fused_adaln_residual_rmsnorm(x, y, None, w, None, None, tokens_per_sample=3)
    assert torch.allclose(h, x + y)
    assert torch.allclose(out, rmsnorm(x + y, w), atol=1e-6)


def test_swiglu_reference():
    a, b = torch.randn(5, 7), torch.randn(5, 7)
    assert torch.allclose(fused_swiglu(a, b), torch.nn.functional.silu(a) * b)
    assert torch.equal(fused_swiglu(a, b), swiglu_ref(a, b))


def test_chunked_ce_cpu_matches_naive():
    torch.manual_seed(1)
    for chunk in (7, 128, 4096):
        hid = torch.randn(50, 12, requires_grad=True)
        w = torch.randn(97, 12, requires_grad=True)
        tgt = torch.randint(0, 97, (50,))
        tgt[::5] = -100
        loss = chunked_cross_entropy(hid, w, tgt, chunk_size=chunk)
        h2, w2 = hid.detach().clone().requires_grad_(True), w.detach().clone().requires_grad_(True)
        ref = chunked_cross_entropy_ref(h2, w2, tgt)
        assert torch.allclose(loss, ref, atol=1e-5)
        loss.backward()
        ref.backward()
        assert torch.allclose(hid.grad, h2.grad, atol=1e-5)
        assert torch.allclose(w.grad, w2.grad, atol=1e-5)
        assert torch.count_nonzero(hid.grad[::5]) == 0


def test_chunked_ce_all_ignored_is_finite():
    hid = torch.randn(8, 4, requires_grad=True)
    w = torch.randn(10, 4, requires_grad=True)
    loss = chunked_cross_entropy(hid, w, torch.full((8,), -100))
    loss.backward()
    assert torch.isfinite(loss) and float(loss) == 0 and torch.count_nonzero(hid.grad) == 0


def test_attention_reference_gqa_and_causal():
    torch.manual_seed(2)
    q = torch.randn(2, 5, 4, 8)
    k = torch.randn(2, 5, 2, 8)
    v = torch.randn(2, 5, 2, 8)
    out = attention(q, k, v, causal=True)
    kk = k.repeat_interleave(2, dim=2)
    vv = v.repeat_interleave(2, dim=2)
    ref = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), kk.transpose(1, 2),
                                                           vv.transpose(1, 2), is_causal=True).transpose(1, 2)
    assert torch.allclose(out, ref, atol=1e-5)
    assert torch.allclose(attention_ref(q.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2)),
                          torch.nn.functional.scaled_dot_product_attention(
                              q.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2)), atol=1e-5)


def test_patchify_matches_conv_layout():
    torch.manual_seed(3)
    img = torch.randint(0, 256, (2, 32, 48, 3), dtype=torch.uint8)
    rows = patchify_images(img, 16, dtype=torch.float32)
    assert rows.shape == (2, 6, 768)
    conv = torch.nn.Conv2d(3, 5, 16, 16)
    chw = normalise_images_ref(img.permute(0, 3, 1, 2), torch.float32)
    ref = conv(chw).flatten(2).transpose(1, 2)
    out = rows @ conv.weight.reshape(5, -1).t() + conv.bias
    assert torch.allclose(out, ref, atol=1e-4)
    assert torch.equal(patchify_ref(img, 16, 776, torch.float32)[..., 768:], torch.zeros(2, 6, 8))


@pytest.mark.parametrize("preset,over", [("ref", {"image_size": 32}), ("tiny", {"image_size": 32})])
def test_model_forward_backward_cpu(preset, over):
    """Both layouts (reference scene-query pooling; BASELINE backbone over image tokens) train on CPU."""
    from nuvla_forge_b200.data import SampleSpec, SyntheticBatchSource
    from nuvla_forge_b200.models import NuVLA, NuVLAConfig

    cfg = NuVLAConfig.preset(preset, fused=False, **over)
    torch.manual_seed(0)
    model = NuVLA(cfg)
    b = SyntheticBatchSource(SampleSpec.for_model(cfg), 2, pin=False).batch(0)
    out = model(b["images"], b["trajectory"], b["text_tokens"], b["text_targets"])
    assert set(out) >= {"loss", "plan_loss", "reason_loss"}
    assert torch.isfinite(out["loss"]) and float(out["loss"]) > 0
    out["loss"].backward()
    grads = [p.grad for p in model.parameters() if p.requires_grad]
    assert sum(g is not None for g in grads) > 0.9 * len(grads)
    assert all(torch.isfinite(g).all() for g in grads if g is not None)


def test_norm_rows_view_alignment():
    """_rows hands the kernels 2-D rows with unit column stride on a 16-byte boundary: aligned
    tensors pass through untouched, misaligned or strided ones are copied."""
    from nuvla_forge_b200.ops.norm import _rows

    n = 64
    t = torch.randn(8, n, dtype=torch.bfloat16)
    assert _rows(t, n) is t
    assert _rows(t.view(2, 4, n), n).data_ptr() == t.data_ptr()
    # a contiguous view that starts 2 bytes into the storage
    flat = torch.randn(8 * n + 1, dtype=torch.bfloat16)
    mis = flat[1:].view(8, n)
    assert mis.is_contiguous() and mis.data_ptr() % 16 != 0
    got = _rows(mis, n)
    assert got.data_ptr() % 16 == 0 and got.is_contiguous() and torch.equal(got, mis)
    # a column slice of a wider tensor: unit stride, rows 16-byte aligned -> read in place
    wide = torch.randn(8, 3 * n, dtype=torch.bfloat16)
    mid = wide[:, n:2 * n]
    assert _rows(mid, n).data_ptr() == mid.data_ptr()
    # a transposed view: copied into packed rows
    tr = torch.randn(n, 8, dtype=torch.bfloat16).t()
    got = _rows(tr, n)
    assert got.stride() == (n, 1) and torch.equal(got, tr)

"""Stack-selective activation checkpointing (train.set_grad_checkpointing) on CPU.

The native model runs its blocks through the fused residual chain (``forward_chain``), so the
checkpoint has to sit inside the blocks: these tests check that every selected block is really
recomputed (counted through torch.utils.checkpoint) and that gradients equal the ones without
checkpointing, on the fused chain and on the unfused blocks.
"""

import pytest
import torch

from nuvla_forge_b200.data import SampleSpec, SyntheticBatchSource
from nuvla_forge_b200.models import NuVLA, NuVLAConfig
from nuvla_forge_b200.train import CHECKPOINT_STACKS, set_grad_checkpointing


def _model(fused: bool):
    cfg = NuVLAConfig.preset("tiny", fused=fused)
    torch.manual_seed(0)
    model = NuVLA(cfg)
    for p in model.dit.out.parameters():  # zero-initialised head: give the DiT blocks a gradient
        torch.nn.init.normal_(p, std=0.1)
    for blk in model.dit.blocks:          # and open the adaLN-Zero gates
        torch.nn.init.normal_(blk.cond[1].weight, std=0.02)
    b = SyntheticBatchSource(SampleSpec.for_model(cfg), 2, pin=False).batch(0)
    return model, b


def _grads(model, b):
    model.zero_grad(set_to_none=True)
    torch.manual_seed(7)  # flow-matching noise and timesteps
    out = model(b["images"], trajectory=b["trajectory"], text_tokens=b["text_tokens"],
                text_targets=b["text_targets"])
    out["loss"].backward()
    return float(out["loss"].detach()), {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}


def _count_checkpoints(monkeypatch):
    calls = []
    real = torch.utils.checkpoint.checkpoint

    def counting(fn, *args, **kw):
        calls.append(getattr(fn, "__self__", None))
        return real(fn, *args, **kw)

    monkeypatch.setattr(torch.utils.checkpoint, "checkpoint", counting)
    return calls


@pytest.mark.parametrize("fused", [True, False])
def test_all_stacks_recomputed_with_equal_gradients(monkeypatch, fused):
    model, b = _model(fused)
    loss0, g0 = _grads(model, b)
    calls = _count_checkpoints(monkeypatch)
    assert set_grad_checkpointing(model, "all") == list(CHECKPOINT_STACKS)
    loss1, g1 = _grads(model, b)
    blocks = (list(model.encoder.blocks) + list(model.fusion) + list(model.text_blocks)
              + list(model.dit.blocks))
    assert set(map(id, blocks)) <= set(map(id, calls)), "a selected block was not checkpointed"
    assert loss1 == pytest.approx(loss0, rel=1e-6, abs=1e-6)
    assert g0.keys() == g1.keys()
    for n in g0:
        torch.testing.assert_close(g1[n], g0[n], rtol=1e-5, atol=1e-6, msg=n)


def test_selection_and_no_grad(monkeypatch):
    model, b = _model(True)
    assert set_grad_checkpointing(model, True) == ["encoder"]
    assert all(blk.grad_checkpoint for blk in model.encoder.blocks)
    assert not any(blk.grad_checkpoint for blk in model.dit.blocks)
    assert set_grad_checkpointing(model, "dit, text") == ["dit", "text"]
    assert not any(blk.grad_checkpoint for blk in model.encoder.blocks)
    assert all(blk.grad_checkpoint for blk in model.dit.blocks)
    assert set_grad_checkpointing(model, None) == []
    assert not any(blk.grad_checkpoint for blk in model.text_blocks)
    with pytest.raises(ValueError):
        set_grad_checkpointing(model, "decoder")
    # no autograd recording: nothing to save, so no checkpoint
    set_grad_checkpointing(model, "all")
    calls = _count_checkpoints(monkeypatch)
    with torch.no_grad():
        model(b["images"], trajectory=b["trajectory"], text_tokens=b["text_tokens"], text_targets=b["text_targets"])
    assert calls == []


def _saved_bytes(model, b):
    """Bytes of the tensors autograd keeps for backward during one forward (storage counted once)."""
    seen = {}

    def pack(t):
        if t.device.type != "meta":
            st = t.untyped_storage()
            seen[st.data_ptr()] = st.nbytes()
        return t

    torch.manual_seed(7)
    with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
        out = model(b["images"], trajectory=b["trajectory"], text_tokens=b["text_tokens"],
                    text_targets=b["text_targets"])
    del out
    return sum(seen.values())


def test_checkpointing_reduces_saved_activations():
    """The chained blocks keep only their inputs: checkpointing every stack cuts the bytes saved
    for backward well below the uncheckpointed forward's (the old wrapper around blk.forward left
    the chained blocks untouched)."""
    model, b = _model(True)
    full = _saved_bytes(model, b)
    set_grad_checkpointing(model, "encoder")
    enc = _saved_bytes(model, b)
    set_grad_checkpointing(model, "all")
    ckpt = _saved_bytes(model, b)
    assert ckpt < enc < full, (full, enc, ckpt)
    assert ckpt < 0.5 * full, (full, ckpt)

"""The fused step leaves the model's saved state as it found it (the reference checks the same,
solution/test_kernels.py:464-486): the adapter file written before installing the step and after
install, a fused training step (forward + backward, no optimizer step) and a fallback call to
the original compute_loss is byte-for-byte the same file, and the base model's NF4 bytes and
absmax (which the step re-points into its own grouped storage) keep their values."""

import types

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _adapter_file(model, path):
    from safetensors.torch import save_file

    names = [n for n, p in model.named_parameters() if p.requires_grad]
    save_file({n: p.detach().contiguous() for n, p in model.named_parameters() if n in names},
              str(path))
    return path.read_bytes()


def _base_state(model):
    out = []
    for layer in model.get_base_model().model.layers:
        for mod in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj,
                    layer.self_attn.o_proj, layer.mlp.gate_proj, layer.mlp.up_proj,
                    layer.mlp.down_proj):
            w = getattr(mod, "base_layer", mod).weight
            out.append((w.data.clone(), w.quant_state.absmax.clone()))
    return out


def test_adapter_and_base_bytes_survive_install_step_and_fallback(tmp_path):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import patch
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import TINY, build_qwen2_qlora

    model = build_qwen2_qlora(TINY, dropout=0.1, device=DEV, seed=5, nested=True)
    model.train()
    before = _adapter_file(model, tmp_path / "before.safetensors")
    base = _base_state(model)
    fallbacks = []

    def original(model_, inputs, return_outputs=False, num_items_in_batch=None):
        fallbacks.append(sorted(inputs))
        return torch.zeros((), device=DEV)

    trainer = types.SimpleNamespace(
        model=model, compute_loss=original, compute_loss_func=None, label_smoother=None,
        model_accepts_loss_kwargs=True, state=types.SimpleNamespace(global_step=0),
        args=types.SimpleNamespace(average_tokens_across_devices=False, n_gpu=1, bf16=False),
        _metrics={"train": {}}, _total_train_tokens=0, _soup_rewind_state=None)
    assert patch.install(trainer)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, TINY.vocab_size, (3, 40), generator=g)
    mask = (torch.arange(40)[None] < torch.tensor([40, 23, 9])[:, None]).long()
    labels = torch.where(mask.bool(), ids, -100)
    inputs = {"input_ids": ids.to(DEV), "attention_mask": mask.to(DEV), "labels": labels.to(DEV)}
    loss = trainer.compute_loss(model, dict(inputs), num_items_in_batch=60)
    loss.backward()
    patch.flush_metrics(trainer)
    assert not fallbacks and torch.isfinite(loss)
    model.eval()  # evaluation: the original compute_loss runs
    trainer.compute_loss(model, dict(inputs))
    assert len(fallbacks) == 1
    torch.cuda.synchronize()
    assert _adapter_file(model, tmp_path / "after.safetensors") == before
    for (packed, absmax), (packed2, absmax2) in zip(base, _base_state(model)):
        assert torch.equal(packed.reshape(-1), packed2.reshape(-1))
        assert torch.equal(absmax, absmax2)


def test_streamed_weights_train_fallback_train():
    """Streamed weights through the drop-in (patch.install(trainer, stream_weights=True)): after
    a fused step the model's 4-bit parameters view pinned host memory; a fallback call to the
    original compute_loss finds them on the GPU with their original bytes (the model's own layers
    can run); the next fused step streams again (the device copy freed) and gives the first
    step's loss bit for bit (the reference's train-eval-train test,
    solution/test_fallback.py:100-117, and its restore_weights, solution/patch.py:280-283)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import patch
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import TINY, build_qwen2_qlora

    model = build_qwen2_qlora(TINY, dropout=0.0, device=DEV, seed=5, nested=True)
    model.train()
    base = _base_state(model)
    seen = []

    def original(model_, inputs, return_outputs=False, num_items_in_batch=None):
        state = _base_state(model_)
        seen.append(all(p.is_cuda and a.is_cuda for p, a in state))
        seen.append(all(torch.equal(p.reshape(-1).cpu(), q.reshape(-1).cpu())
                        and torch.equal(a.cpu(), b.cpu()) for (p, a), (q, b) in zip(state, base)))
        return torch.zeros((), device=DEV)

    trainer = types.SimpleNamespace(
        model=model, compute_loss=original, compute_loss_func=None, label_smoother=None,
        model_accepts_loss_kwargs=True, state=types.SimpleNamespace(global_step=0),
        args=types.SimpleNamespace(average_tokens_across_devices=False, n_gpu=1, bf16=False),
        _metrics={"train": {}}, _total_train_tokens=0, _soup_rewind_state=None)
    assert patch.install(trainer, stream_weights=True)
    engine = getattr(trainer, patch._INSTALLED_ATTR)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, TINY.vocab_size, (3, 40), generator=g)
    mask = (torch.arange(40)[None] < torch.tensor([40, 23, 9])[:, None]).long()
    labels = torch.where(mask.bool(), ids, -100)
    inputs = {"input_ids": ids.to(DEV), "attention_mask": mask.to(DEV), "labels": labels.to(DEV)}
    losses = []

    def fused():
        loss = trainer.compute_loss(model, dict(inputs), num_items_in_batch=60)
        loss.backward()
        patch.flush_metrics(trainer)
        losses.append(loss.detach())

    fused()
    assert all(not p.is_cuda and not a.is_cuda for p, a in _base_state(model))
    model.eval()  # evaluation: the original compute_loss runs the model's own layers
    trainer.compute_loss(model, dict(inputs))
    model.train()
    assert seen == [True, True]
    assert engine.wstream.device_copy is not None
    fused()
    assert engine.wstream.device_copy is None
    assert all(not p.is_cuda and not a.is_cuda for p, a in _base_state(model))
    torch.cuda.synchronize()
    assert torch.isfinite(losses[0]) and torch.equal(losses[0], losses[1])

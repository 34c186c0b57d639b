"""The drop-in boundary: `fused_compute_loss` replaces an HF Trainer's `compute_loss` with the
fused B200 step and keeps the trainer's own bookkeeping (solution/patch.py:268-389 of the
reference): same inputs, same loss normalisation, same TRL metrics (entropy, mean token accuracy,
num_tokens) and Soup rewind rows, same fallback to the original code for anything the fused step
does not take. HF Trainer, its optimizer, GradScaler and LR schedule are untouched.

    from hack_fe30cb28_opus_5_5_ultracode_b200 import patch
    patch.install(trainer)          # True if the model is a supported QLoRA Qwen2

bitsandbytes and peft are not required: the support check reads the model duck-typed (a 4-bit
projection is any module whose weight has an NF4 `quant_state`).
"""

import sys
import types

import torch

_INSTALLED_ATTR = "_soup_kernels_engine"


def _log(message):
    print(f"[qlora-b200] {message}", file=sys.stderr, flush=True)


def _is_nf4(module):
    base = getattr(module, "base_layer", module)
    state = getattr(getattr(base, "weight", None), "quant_state", None)
    return state is not None and getattr(state, "quant_type", None) == "nf4"


def is_supported(model):
    """Qwen2 + silu + default RoPE, every projection NF4, LoRA (one active adapter, no DoRA) on
    q_proj and v_proj only (solution/patch.py:154-203)."""
    if not isinstance(model, torch.nn.Module) or not hasattr(model, "get_base_model"):
        return False
    causal = model.get_base_model()
    config = getattr(causal, "config", None)
    if getattr(config, "model_type", None) != "qwen2" or getattr(config, "hidden_act", "") != "silu":
        return False
    if getattr(config, "use_sliding_window", False):
        return False
    rope = getattr(config, "rope_parameters", None) or getattr(config, "rope_scaling", None) or {}
    if (rope.get("rope_type", rope.get("type", "default")) or "default") != "default":
        return False
    inner = getattr(causal, "model", None)
    if inner is None or not hasattr(inner, "layers"):
        return False
    if not torch.cuda.is_available() or inner.norm.weight.device.type != "cuda":
        return False
    if getattr(config, "head_dim", None) not in (None, 128) and \
            config.hidden_size // config.num_attention_heads != 128:
        return False
    for layer in inner.layers:
        attn, mlp = layer.self_attn, layer.mlp
        for name, module in (("q_proj", attn.q_proj), ("k_proj", attn.k_proj),
                             ("v_proj", attn.v_proj), ("o_proj", attn.o_proj),
                             ("gate_proj", mlp.gate_proj), ("up_proj", mlp.up_proj),
                             ("down_proj", mlp.down_proj)):
            if not _is_nf4(module):
                return False
            if hasattr(module, "lora_A"):
                if name not in ("q_proj", "v_proj") or getattr(module, "merged", False) \
                        or getattr(module, "disable_adapters", False):
                    return False
                active = list(getattr(module, "active_adapters", []))
                if len(active) != 1 or active[0] not in module.lora_A:
                    return False
                if getattr(module, "use_dora", {}).get(active[0], False):
                    return False
            elif name in ("q_proj", "v_proj"):
                return False
    return True


def fused_compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
    """Trainer.compute_loss with the fused step (solution/patch.py:268-346)."""
    engine = getattr(self, _INSTALLED_ATTR, None)
    original = getattr(self, "_soup_original_compute_loss")
    usable = (
        engine is not None
        and getattr(model, "training", False)
        and isinstance(inputs, dict)
        and set(inputs) <= {"input_ids", "attention_mask", "labels", "_prediction_loss_only"}
        and all(key in inputs for key in ("input_ids", "attention_mask", "labels"))
        and getattr(self, "compute_loss_func", None) is None
        and getattr(self, "label_smoother", None) is None
    )
    if not usable:
        return original(model, inputs, return_outputs=return_outputs,
                        num_items_in_batch=num_items_in_batch)
    popped = {key: inputs.pop(key) for key in ("_prediction_loss_only",) if key in inputs}
    input_ids, attention_mask, labels = (inputs["input_ids"], inputs["attention_mask"],
                                         inputs["labels"])
    # HF Trainer: sum over the batch / num_items_in_batch when the model takes loss kwargs,
    # otherwise the model's mean over supervised tokens.
    if getattr(self, "model_accepts_loss_kwargs", False) and num_items_in_batch is not None:
        denom = num_items_in_batch
    else:
        denom = (labels[:, 1:] != -100).sum()
    denom = float(denom.item() if torch.is_tensor(denom) else denom)
    from .engine import UnsupportedBatch

    host = getattr(self, "_qlora_host_batch", None)
    self._qlora_host_batch = None
    if host is not None and (host[0] is not input_ids):
        host = None  # stale: prepared for other inputs
    try:
        loss, packed, stats = engine.step(input_ids, attention_mask, labels, denom,
                                          host[1] if host is not None else None)
    except UnsupportedBatch:  # raised before the step changed anything
        inputs.update(popped)
        return original(model, inputs, return_outputs=return_outputs,
                        num_items_in_batch=num_items_in_batch)
    args = getattr(self, "args", None)
    if getattr(args, "average_tokens_across_devices", False) \
            and getattr(self, "model_accepts_loss_kwargs", False) and num_items_in_batch is not None:
        accel = getattr(self, "accelerator", None)
        scale = getattr(accel, "num_processes", 1)
        pc = getattr(accel, "parallelism_config", None)
        if pc is not None:
            scale //= pc.tp_size
        loss = loss * (scale if getattr(args, "n_gpu", 1) <= 1 else args.n_gpu)

    # TRL metrics and Soup's rewind rows, recorded once backward is queued (no host sync between
    # forward and backward): same values, same order as TRL's / Soup's own compute_loss.
    _flush_metrics(self)
    metrics = self._metrics["train"]
    metrics["entropy"], metrics["mean_token_accuracy"]  # noqa: B018 - keys in TRL's order
    self._total_train_tokens += int(packed.n)
    metrics["num_tokens"] = [self._total_train_tokens]
    self._soup_pending_metrics = (packed, stats, labels, int(self.state.global_step) + 1)
    if return_outputs:
        try:
            from transformers.modeling_outputs import CausalLMOutputWithPast

            return loss, CausalLMOutputWithPast(loss=loss, logits=None)
        except ImportError:
            return loss, types.SimpleNamespace(loss=loss, logits=None)
    return loss


def prepare_inputs(trainer, inputs, device):
    """Move a host batch to the GPU as HF Trainer._prepare_inputs does (pinned, non-blocking)
    and keep its HostBatch (lengths, supervised count) for the next fused_compute_loss, which
    then reads nothing back from the device. install() routes the trainer's own
    _prepare_inputs through this."""
    from .engine import HostBatch

    host = None
    if isinstance(inputs, dict) and "attention_mask" in inputs and "labels" in inputs \
            and not inputs["attention_mask"].is_cuda and not inputs["labels"].is_cuda:
        host = HostBatch.of(inputs["attention_mask"], inputs["labels"])
    device = torch.device(device)

    def move(v):
        if not torch.is_tensor(v) or v.device == device:
            return v
        if device.type == "cuda":
            return v.pin_memory().to(device, non_blocking=True)
        return v.to(device)

    moved = {k: move(v) for k, v in inputs.items()}
    if host is not None and "input_ids" in moved:
        trainer._qlora_host_batch = (moved["input_ids"], host)
    return moved


def _flush_metrics(trainer):
    """Record the queued micro-batch's TRL metrics and Soup rewind row
    (solution/patch.py:349-389)."""
    pending = getattr(trainer, "_soup_pending_metrics", None)
    if pending is None:
        return
    trainer._soup_pending_metrics = None
    packed, stats, labels, step = pending
    with torch.no_grad():
        valid = packed.targets >= 0
        summary = torch.stack([stats.entropy.sum(), stats.correct.sum().float(),
                               valid.sum().float()]).tolist()
    trainer._metrics["train"]["entropy"].append(summary[0] / max(packed.n, 1))
    trainer._metrics["train"]["mean_token_accuracy"].append(
        summary[1] / summary[2] if summary[2] > 0 else 0.0)
    state = getattr(trainer, "_soup_rewind_state", None)
    if state is not None and not state.failed:
        try:
            with torch.no_grad():
                totals = torch.zeros(packed.rows, device=labels.device, dtype=torch.float32)
                totals.index_add_(0, packed.row_of_token.index_select(0, stats.order),
                                  stats.tok_loss)
                counts = (labels[:, 1:] != -100).sum(dim=1)
                means = totals / counts.clamp(min=1).to(totals.dtype)
            state.on_micro_batch(step=step, row_loss=[float(x) for x in means.tolist()],
                                 row_tokens=[int(x) for x in counts.tolist()])
        except Exception as exc:  # noqa: BLE001 - the recorder never raises into training
            state.fail(exc)


def _callback_base():
    try:
        import transformers

        return transformers.TrainerCallback
    except ImportError:  # pragma: no cover
        return object


class _FlushMetrics(_callback_base()):
    def __init__(self, trainer):
        self.trainer = trainer

    def on_pre_optimizer_step(self, args, state, control, **kwargs):
        _flush_metrics(self.trainer)

    def on_step_end(self, args, state, control, **kwargs):
        _flush_metrics(self.trainer)


def install(trainer, dtype=None):
    """Installs the fused step as trainer.compute_loss if the model is supported; returns
    whether it did (solution/patch.py:452-503). dtype: the compute type, from the trainer's
    args (bf16 / fp16) unless given."""
    model = getattr(trainer, "model", None)
    if getattr(trainer, _INSTALLED_ATTR, None) is not None:
        return True
    if not is_supported(model):
        _log("model not recognized, training with the original code path")
        return False
    from .engine import FusedQwen2

    if dtype is None:
        args = getattr(trainer, "args", None)
        dtype = torch.bfloat16 if getattr(args, "bf16", False) else torch.float16
    engine = FusedQwen2(model, dtype=dtype)
    trainer._soup_original_compute_loss = trainer.compute_loss
    setattr(trainer, _INSTALLED_ATTR, engine)
    trainer.compute_loss = types.MethodType(fused_compute_loss, trainer)
    original_prepare = getattr(trainer, "_prepare_inputs", None)
    if original_prepare is not None:
        def _prepare_inputs(inputs):
            # keep the batch's host-side facts before HF moves it (no device read-backs later)
            from .engine import HostBatch

            host = None
            if isinstance(inputs, dict) and "attention_mask" in inputs and "labels" in inputs \
                    and torch.is_tensor(inputs["attention_mask"]) \
                    and not inputs["attention_mask"].is_cuda and not inputs["labels"].is_cuda:
                host = HostBatch.of(inputs["attention_mask"], inputs["labels"])
            moved = original_prepare(inputs)
            if host is not None and isinstance(moved, dict) and "input_ids" in moved:
                trainer._qlora_host_batch = (moved["input_ids"], host)
            return moved

        trainer._prepare_inputs = _prepare_inputs
    if hasattr(trainer, "add_callback"):
        trainer.add_callback(_FlushMetrics(trainer))
    _log(f"fused Qwen2 step installed ({len(engine.layers)} layers, {dtype}, LoRA dropout "
         f"{engine.dropout_p})")
    return True


def apply():
    """Patch soup_cli's SFT trainer wrapper so every Soup run installs the fused step when it
    starts training (solution/__init__.py:11-31); a no-op without soup_cli."""
    try:
        from soup_cli.trainer import sft  # noqa: F401
    except Exception:  # noqa: BLE001
        _log("soup_cli not importable: call patch.install(trainer) yourself")
        return False
    wrapper = sft.SFTTrainerWrapper
    if getattr(wrapper, "_qlora_b200_patched", False):
        return True
    original_train = wrapper.train

    def train(self, *args, **kwargs):
        trainer = getattr(self, "trainer", None)
        if trainer is not None:
            try:
                install(trainer)
            except Exception as exc:  # noqa: BLE001 - anything unexpected: original code path
                _log(f"install failed ({exc!r}); training with the original code path")
        return original_train(self, *args, **kwargs)

    wrapper.train = train
    wrapper._qlora_b200_patched = True
    return True

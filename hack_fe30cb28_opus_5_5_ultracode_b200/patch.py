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

_INSTALLED_ATTR = "_qlora_b200_step"      # the FusedQwen2 an installed trainer runs
_ORIGINAL_ATTR = "_qlora_b200_original"   # the trainer's own compute_loss


def _log(message):
    print(f"[qlora-b200] {message}", file=sys.stderr, flush=True)


def _is_nf4(module):
    base = getattr(module, "base_layer", module)
    state = getattr(getattr(base, "weight", None), "quant_state", None)
    return state is not None and getattr(state, "quant_type", None) == "nf4"


def is_supported(model):
    """Qwen2 + silu + default RoPE, every projection NF4, LoRA (one active adapter, no DoRA) on
    q_proj and v_proj only (solution/patch.py:154-203), heads of 64 or 128."""
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
    head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
    if head_dim not in (64, 128):  # the attention kernels of this library
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


_ACCEPTED_KEYS = frozenset({"input_ids", "attention_mask", "labels", "_prediction_loss_only"})
_REQUIRED_KEYS = ("input_ids", "attention_mask", "labels")


def _why_not_fused(trainer, model, inputs):
    """None when the fused step can take this compute_loss call, else the reason it cannot (the
    original code then runs). The fused step covers plain causal-LM training on a right-padded
    batch: no eval pass, no extra model inputs, no custom loss or label smoothing
    (solution/patch.py:268-285 draws the same line)."""
    if getattr(trainer, _INSTALLED_ATTR, None) is None:
        return "not installed"
    if not getattr(model, "training", False):
        return "evaluation"
    if not isinstance(inputs, dict) or not set(inputs) <= _ACCEPTED_KEYS \
            or any(key not in inputs for key in _REQUIRED_KEYS):
        return "inputs other than input_ids / attention_mask / labels"
    if getattr(trainer, "compute_loss_func", None) is not None:
        return "a custom loss function"
    if getattr(trainer, "label_smoother", None) is not None:
        return "label smoothing"
    return None


def _loss_denominator(trainer, labels, num_items_in_batch):
    """What HF Trainer divides the summed token losses by: the trainer's own token count when
    the model takes loss kwargs, else the number of shifted labels with a target (the model's
    mean loss)."""
    if num_items_in_batch is not None and getattr(trainer, "model_accepts_loss_kwargs", False):
        count = num_items_in_batch
    else:
        count = (labels[..., 1:] != -100).sum()
    return float(count.item()) if torch.is_tensor(count) else float(count)


def _cross_device_factor(trainer, num_items_in_batch):
    """HF Trainer's multiplier of the loss under average_tokens_across_devices: its token count
    covers every process, and the gradient all-reduce averages, so the loss is scaled by the
    number of data-parallel replicas (processes over the tensor-parallel size, or n_gpu under
    DataParallel)."""
    args = getattr(trainer, "args", None)
    if num_items_in_batch is None or not getattr(args, "average_tokens_across_devices", False) \
            or not getattr(trainer, "model_accepts_loss_kwargs", False):
        return 1
    n_gpu = getattr(args, "n_gpu", 1)
    if n_gpu > 1:
        return n_gpu
    accelerator = getattr(trainer, "accelerator", None)
    replicas = getattr(accelerator, "num_processes", 1)
    parallelism = getattr(accelerator, "parallelism_config", None)
    return replicas // parallelism.tp_size if parallelism is not None else replicas


class MetricLedger:
    """The logged side effects of fused steps, kept until the trainer's next optimizer step:
    TRL's `entropy` (mean over a micro-batch's real tokens) and `mean_token_accuracy` (over the
    tokens with a target), and Soup's rewind row (each row's mean cross-entropy over its
    targets). `record` reduces one small summary per micro-batch on the GPU right after the
    step and starts its copy into pinned host memory on the same stream (no host sync between
    forward and backward); `flush` waits for those copies - done long before, as the head of
    each forward finished - and appends the values in micro-batch order, before the optimizer
    step and the log read them (solution/patch.py:334-389 keeps the same values). The flush
    therefore does not wait for the backward, and the optimizer's launches are not held back
    behind it. The pinned host buffers are reused from flush to flush (pinning memory on every
    step could wait for the GPU's queued work)."""

    def __init__(self):
        self.pending = []  # (summary: host copy or tensor, copy event, rows, real tokens, step)
        self.free = []     # pinned float64 buffers the last flush gave back
        self.lent = []     # the buffers of the pending summaries

    def _pinned(self, n):
        for k, buf in enumerate(self.free):
            if buf.numel() >= n:
                del self.free[k]
                break
        else:
            buf = torch.empty(max(64, 2 * n), dtype=torch.float64, pin_memory=True)
        self.lent.append(buf)
        return buf[:n]

    def record(self, packed, stats, labels, step):
        rows = packed.rows
        with torch.no_grad():
            row_of = packed.row_of_token.index_select(0, stats.order)
            per_row = torch.zeros(rows, device=stats.tok_loss.device, dtype=torch.float64)
            per_row.index_add_(0, row_of, stats.tok_loss.double())
            row_targets = (labels[:, 1:] != -100).sum(dim=1).double().to(per_row.device)
            head = torch.stack([stats.entropy.double().sum(), stats.correct.double().sum(),
                                (packed.targets >= 0).double().sum()])
            summary = torch.cat([head, per_row, row_targets])
            done = None
            if summary.is_cuda:
                host = self._pinned(summary.numel())
                host.copy_(summary, non_blocking=True)
                done = torch.cuda.Event()
                done.record()
                summary = host
        self.pending.append((summary, done, rows, packed.n, step))

    def flush(self, trainer):
        if not self.pending:
            return
        pending, self.pending = self.pending, []
        for _, done, _, _, _ in pending:
            if done is not None:
                done.synchronize()
        values = torch.cat([s for s, _, _, _, _ in pending]).tolist()
        self.free.extend(self.lent)
        self.lent = []
        metrics = trainer._metrics["train"]
        recorder = getattr(trainer, "_soup_rewind_state", None)
        at = 0
        for _, _, rows, real, step in pending:
            ent, correct, supervised = values[at:at + 3]
            per_row = values[at + 3:at + 3 + rows]
            targets = values[at + 3 + rows:at + 3 + 2 * rows]
            at += 3 + 2 * rows
            metrics["entropy"].append(ent / max(real, 1.0))
            metrics["mean_token_accuracy"].append(correct / supervised if supervised else 0.0)
            if recorder is None or recorder.failed:
                continue
            try:  # the rewind recorder must never stop training
                recorder.on_micro_batch(step=step,
                                        row_loss=[s / max(c, 1.0) for s, c in zip(per_row, targets)],
                                        row_tokens=[int(c) for c in targets])
            except Exception as exc:  # noqa: BLE001
                recorder.fail(exc)


def ledger(trainer):
    """The trainer's MetricLedger (made on first use)."""
    book = getattr(trainer, "_qlora_ledger", None)
    if book is None:
        book = trainer._qlora_ledger = MetricLedger()
    return book


def flush_metrics(trainer):
    """Appends every queued micro-batch's TRL metrics and Soup rewind rows (see MetricLedger)."""
    ledger(trainer).flush(trainer)


def _run_original(trainer, model, inputs, return_outputs, num_items_in_batch):
    engine = getattr(trainer, _INSTALLED_ATTR, None)
    if engine is not None and hasattr(engine, "restore_weights"):
        engine.restore_weights()  # the original code runs the 4-bit layers: weights on the GPU
    return getattr(trainer, _ORIGINAL_ATTR)(model, inputs, return_outputs=return_outputs,
                                            num_items_in_batch=num_items_in_batch)


def fused_compute_loss(self, model, inputs, return_outputs=False, num_items_in_batch=None):
    """HF Trainer.compute_loss through the fused step (the hook the reference installs,
    solution/patch.py:268-346): the loss is the summed token cross-entropy over HF's
    denominator, scaled for cross-device averaging; the step's LoRA gradients reach PEFT's
    parameters through autograd; TRL's metrics and Soup's rewind rows are queued for the next
    optimizer step. Anything the step does not take runs the trainer's original compute_loss."""
    if _why_not_fused(self, model, inputs) is not None:
        return _run_original(self, model, inputs, return_outputs, num_items_in_batch)
    labels = inputs["labels"]
    denom = _loss_denominator(self, labels, num_items_in_batch)
    staged = getattr(self, "_qlora_host_batch", None)
    self._qlora_host_batch = None
    host = staged[1] if staged is not None and staged[0] is inputs["input_ids"] else None
    from .engine import UnsupportedBatch

    step = getattr(self, _INSTALLED_ATTR)
    try:
        loss, packed, stats = step.step(inputs["input_ids"], inputs["attention_mask"], labels,
                                        denom, host)
    except UnsupportedBatch:  # raised before the step changed any state
        return _run_original(self, model, inputs, return_outputs, num_items_in_batch)
    factor = _cross_device_factor(self, num_items_in_batch)
    if factor != 1:
        loss = loss * factor
    metrics = self._metrics["train"]
    for key in ("entropy", "mean_token_accuracy"):  # TRL creates these two before num_tokens
        metrics.setdefault(key, [])
    self._total_train_tokens += int(packed.n)
    metrics["num_tokens"] = [self._total_train_tokens]
    ledger(self).record(packed, stats, labels, int(self.state.global_step) + 1)
    if not return_outputs:
        return loss
    try:
        from transformers.modeling_outputs import CausalLMOutputWithPast

        return loss, CausalLMOutputWithPast(loss=loss, logits=None)
    except ImportError:
        return loss, types.SimpleNamespace(loss=loss, logits=None)


def _host_facts(inputs):
    """The HostBatch of a batch still in host memory (None for anything else)."""
    from .engine import HostBatch

    if not isinstance(inputs, dict):
        return None
    mask, labels, ids = inputs.get("attention_mask"), inputs.get("labels"), inputs.get("input_ids")
    if not (torch.is_tensor(mask) and torch.is_tensor(labels)) or mask.is_cuda or labels.is_cuda:
        return None
    return HostBatch.of(mask, labels, ids if torch.is_tensor(ids) and not ids.is_cuda else None)


def prepare_inputs(trainer, inputs, device):
    """Moves a host batch to the GPU as HF Trainer._prepare_inputs does (non-blocking: pinned
    tensors directly, others through the engine's reusable pinned staging buffers) and keeps its
    HostBatch for the next fused_compute_loss, which then reads nothing back from the device."""
    from .engine import staging

    host = _host_facts(inputs)
    device = torch.device(device)

    def move(v):
        if not torch.is_tensor(v) or v.device == device:
            return v
        if device.type != "cuda" or v.device.type != "cpu":
            return v.to(device)
        if v.is_pinned():
            return v.to(device, non_blocking=True)
        return staging(device).tensor_to_device(v, device)

    moved = {k: move(v) for k, v in inputs.items()}
    if host is not None and "input_ids" in moved:
        trainer._qlora_host_batch = (moved["input_ids"], host)
    return moved


def _callback_base():
    try:
        import transformers

        return transformers.TrainerCallback
    except ImportError:  # pragma: no cover
        return object


class _LedgerFlush(_callback_base()):
    """Writes the queued metrics before each optimizer step (and at a step's end, for a step
    that ran no optimizer step)."""

    def __init__(self, trainer):
        self.trainer = trainer

    def on_pre_optimizer_step(self, args, state, control, **kwargs):
        flush_metrics(self.trainer)

    def on_step_end(self, args, state, control, **kwargs):
        flush_metrics(self.trainer)


def install(trainer, dtype=None, **engine_options):
    """Installs the fused step as trainer.compute_loss if the model is supported; returns
    whether it did (solution/patch.py:452-503). dtype: the compute type, from the trainer's
    args (bf16 / fp16) unless given; engine_options: FusedQwen2's memory options
    (stream_weights, spill, activation_budget_mib, step_budget_mib, keep_weights, ...)."""
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
    engine = FusedQwen2(model, dtype=dtype, **engine_options)
    setattr(trainer, _ORIGINAL_ATTR, trainer.compute_loss)
    setattr(trainer, _INSTALLED_ATTR, engine)
    trainer.compute_loss = types.MethodType(fused_compute_loss, trainer)
    original_prepare = getattr(trainer, "_prepare_inputs", None)
    if original_prepare is not None:
        def _prepare_inputs(inputs):
            # the batch's host-side facts, taken before HF moves it (no device reads later)
            host = _host_facts(inputs)
            moved = original_prepare(inputs)
            if host is not None and isinstance(moved, dict) and "input_ids" in moved:
                trainer._qlora_host_batch = (moved["input_ids"], host)
            return moved

        trainer._prepare_inputs = _prepare_inputs
    if hasattr(trainer, "add_callback"):
        trainer.add_callback(_LedgerFlush(trainer))
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

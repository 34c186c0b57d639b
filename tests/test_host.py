"""CPU: host-side logic of the fused step — batch packing, the dropout-call arithmetic, the
model stand-in, and the drop-in boundary's bookkeeping and fallbacks (solution/test_fallback.py
is the reference's model for the latter: a SimpleNamespace trainer, the original compute_loss
called for anything the fused step does not take)."""

import types

import numpy as np
import pytest
import torch

from hack_fe30cb28_opus_5_5_ultracode_b200 import patch
from hack_fe30cb28_opus_5_5_ultracode_b200.engine import (HeadStats, Packed, RopeTable,
                                                          UnsupportedBatch, dropout_call)
from hack_fe30cb28_opus_5_5_ultracode_b200.model import TINY, build_qwen2_qlora
from oracle.philox import draw


def _batch(lengths, left=False, vocab=3000, prompt=2):
    torch.manual_seed(3)
    B, T = len(lengths), max(lengths)
    ids = torch.randint(0, vocab, (B, T))
    ar = torch.arange(T)[None]
    L = torch.tensor(lengths)[:, None]
    mask = ((ar >= T - L) if left else (ar < L)).long()
    labels = torch.where(mask.bool(), ids, -100)
    labels[:, :prompt] = -100
    return {"input_ids": ids, "attention_mask": mask, "labels": labels}


def test_packed_unpads_and_shifts():
    b = _batch([5, 3, 7])
    p = Packed(b["input_ids"], b["attention_mask"], b["labels"])
    assert p.n == 15 and p.rows == 3 and p.T == 7 and p.max_len == 7
    assert p.cu_seqlens.tolist() == [0, 5, 8, 15]
    assert p.tok.tolist() == [0, 1, 2, 3, 4, 7, 8, 9, 14, 15, 16, 17, 18, 19, 20]
    assert p.pos.tolist() == [0, 1, 2, 3, 4, 0, 1, 2, 0, 1, 2, 3, 4, 5, 6]
    assert torch.equal(p.ids, b["input_ids"].reshape(-1)[p.tok])
    # targets: the next token's label (HF labels are unshifted), -100 at each row's end
    lab = b["labels"]
    exp = []
    for r, ln in enumerate([5, 3, 7]):
        exp += [int(lab[r, t + 1]) for t in range(ln - 1)] + [-100]
    assert p.targets.tolist() == exp
    sup = [t >= 0 for t in exp]
    assert p.n_supervised == sum(sup)
    order = p.head_order.tolist()
    assert all(sup[i] for i in order[:p.n_supervised]) and not any(sup[i] for i in order[p.n_supervised:])
    assert order[:p.n_supervised] == sorted(order[:p.n_supervised])  # stable
    assert p.row_of_token.tolist() == [0] * 5 + [1] * 3 + [2] * 7


def test_packed_rejects_left_padding_and_bad_shapes():
    b = _batch([5, 3], left=True)
    with pytest.raises(UnsupportedBatch):
        Packed(b["input_ids"], b["attention_mask"], b["labels"])
    with pytest.raises(UnsupportedBatch):
        Packed(b["input_ids"][0], b["attention_mask"][0], b["labels"][0])


@pytest.mark.parametrize("nelem,max_blocks", [(4 * 512 * 1536, 1184), (960, 1184), (8, 1184),
                                              (4 * 37 * 1536, 160), (10**9, 1184)])
def test_dropout_call_matches_oracle(nelem, max_blocks):
    threads, inc = dropout_call(nelem, max_blocks)
    _, ctr, thr, off = draw(nelem, 40, 5, max_blocks)
    assert (threads, 40 + inc, ctr) == (thr, off, 10)


def test_rope_table_is_rotate_half():
    model = build_qwen2_qlora(TINY, device="cpu", seed=0)
    table = RopeTable(model.get_base_model().model.rotary_emb, TINY.head_dim, "cpu")
    cos, sin = table.table(300)
    assert cos.shape == (1024, TINY.head_dim // 2)
    inv = 1.0 / (TINY.rope_theta ** (torch.arange(0, TINY.head_dim, 2).float() / TINY.head_dim))
    torch.testing.assert_close(cos[7], torch.cos(7 * inv))
    assert table.table(2000)[0].shape[0] == 2048


def test_model_stand_in_has_the_peft_bnb_layout():
    model = build_qwen2_qlora(TINY, device="cpu", seed=0, nested=True)
    causal = model.get_base_model()
    layer = causal.model.layers[0]
    q = layer.self_attn.q_proj
    assert q.base_layer.weight.quant_state.quant_type == "nf4"
    assert q.base_layer.weight.data.dtype == torch.uint8
    assert q.base_layer.weight.data.numel() * 2 == TINY.num_attention_heads * TINY.head_dim * TINY.hidden_size
    assert q.lora_A["default"].weight.requires_grad and q.scaling["default"] == 2.0
    assert not hasattr(layer.self_attn.k_proj, "lora_A")
    assert causal.lm_head.weight is causal.model.embed_tokens.weight
    params = [p for p in model.parameters() if p.requires_grad]
    assert len(params) == 4 * TINY.num_hidden_layers
    assert patch.is_supported(model) is False  # no GPU here: the fused step is never offered


# ---------------------------------------------------------------------------------------------
# the boundary (solution/patch.py:268-389), with a stand-in engine
# ---------------------------------------------------------------------------------------------
class _FakeEngine:
    """Runs Packed on the batch and returns a loss with the fused step's statistics."""

    def __init__(self, fail=False):
        self.calls, self.fail = [], fail
        self.restored = 0  # restore_weights calls (before each run of the original code)

    def restore_weights(self):
        self.restored += 1

    def step(self, input_ids, attention_mask, labels, denom, host=None):
        self.calls.append(denom)
        packed = Packed(input_ids, attention_mask, labels, host)  # raises UnsupportedBatch itself
        if self.fail:
            raise UnsupportedBatch("dropout masks differ")
        n = packed.n
        stats = HeadStats()
        stats.order = packed.head_order
        stats.tok_loss = torch.where(packed.targets[stats.order] >= 0, torch.ones(n) * 2.0,
                                     torch.zeros(n))
        stats.entropy = torch.full((n,), 3.0)
        stats.correct = (torch.arange(n) % 2 == 0).int() * (packed.targets[stats.order] >= 0).int()
        loss = stats.tok_loss.sum() / denom
        return loss, packed, stats


class _Rewind:
    def __init__(self):
        self.rows, self.failed = [], False

    def on_micro_batch(self, step, row_loss, row_tokens):
        self.rows.append((step, row_loss, row_tokens))

    def fail(self, exc):
        self.failed = True


def _trainer(engine, **kw):
    calls = []

    def original(model, inputs, return_outputs=False, num_items_in_batch=None):
        calls.append(sorted(inputs))
        return torch.tensor(123.0)

    t = types.SimpleNamespace(compute_loss_func=None, label_smoother=None,
                              model_accepts_loss_kwargs=True,
                              args=types.SimpleNamespace(average_tokens_across_devices=False,
                                                         n_gpu=1),
                              state=types.SimpleNamespace(global_step=4),
                              _metrics={"train": {"entropy": [], "mean_token_accuracy": [],
                                                  "num_tokens": []}},
                              _total_train_tokens=0, _soup_rewind_state=_Rewind())
    setattr(t, patch._ORIGINAL_ATTR, original)
    setattr(t, patch._INSTALLED_ATTR, engine)
    for k, v in kw.items():
        setattr(t, k, v)
    return t, calls


class _Model(torch.nn.Module):
    pass


def test_fused_compute_loss_bookkeeping():
    engine = _FakeEngine()
    t, calls = _trainer(engine)
    model = _Model().train()
    b = _batch([5, 3, 7])
    n_items = int((b["labels"][:, 1:] != -100).sum())
    loss = patch.fused_compute_loss(t, model, dict(b), num_items_in_batch=torch.tensor(n_items))
    assert not calls and engine.calls == [float(n_items)]
    assert loss.item() == pytest.approx(2.0)  # every supervised token costs 2
    assert t._total_train_tokens == 15 and t._metrics["train"]["num_tokens"] == [15]
    patch.flush_metrics(t)
    assert t._metrics["train"]["entropy"] == [pytest.approx(3.0)]
    sup = n_items
    assert t._metrics["train"]["mean_token_accuracy"][0] == pytest.approx(
        sum(1 for i in range(15) if i % 2 == 0 and i < sup) / sup)
    (step, row_loss, row_tokens), = t._soup_rewind_state.rows
    assert step == 5 and row_tokens == [3, 1, 5] and row_loss == [2.0, 2.0, 2.0]
    # without loss kwargs the denominator is the supervised count
    t2, _ = _trainer(_FakeEngine(), model_accepts_loss_kwargs=False)
    patch.fused_compute_loss(t2, model, dict(b), num_items_in_batch=99)
    assert getattr(t2, patch._INSTALLED_ATTR).calls == [float(n_items)]


def test_fused_compute_loss_scales_under_average_tokens_across_devices():
    t, _ = _trainer(_FakeEngine())
    t.args.average_tokens_across_devices = True
    t.accelerator = types.SimpleNamespace(num_processes=4, parallelism_config=None)
    model = _Model().train()
    b = _batch([5, 3, 7])
    n_items = int((b["labels"][:, 1:] != -100).sum())
    loss = patch.fused_compute_loss(t, model, dict(b), num_items_in_batch=n_items)
    assert loss.item() == pytest.approx(8.0)


@pytest.mark.parametrize("case", ["eval", "extra_key", "label_smoother", "left_padding",
                                  "unsupported_batch"])
def test_fused_compute_loss_falls_back(case):
    engine = _FakeEngine(fail=case == "unsupported_batch")
    t, calls = _trainer(engine)
    model = _Model().train()
    b = _batch([5, 3], left=case == "left_padding")
    b["_prediction_loss_only"] = False
    if case == "eval":
        model.eval()
    if case == "extra_key":
        b["position_ids"] = torch.zeros_like(b["input_ids"])
    if case == "label_smoother":
        t.label_smoother = object()
    loss = patch.fused_compute_loss(t, model, b, num_items_in_batch=3)
    assert loss.item() == 123.0 and len(calls) == 1
    assert engine.restored == 1  # the original code runs the model's own layers
    assert "_prediction_loss_only" in calls[0]  # the inputs reach the original unchanged
    assert t._total_train_tokens == 0


def test_install_refuses_unsupported_models():
    t = types.SimpleNamespace(model=_Model(), compute_loss=lambda *a, **k: None)
    assert patch.install(t) is False
    assert not hasattr(t, patch._INSTALLED_ATTR) or getattr(t, patch._INSTALLED_ATTR) is None


def test_host_batch_matches_the_device_reads():
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import HostBatch

    b = _batch([5, 3, 7])
    host = HostBatch.of(b["attention_mask"], b["labels"])
    a = Packed(b["input_ids"], b["attention_mask"], b["labels"])
    p = Packed(b["input_ids"], b["attention_mask"], b["labels"], host)
    assert host.lengths == [5, 3, 7] and host.n_supervised == a.n_supervised == p.n_supervised
    for name in ("tok", "pos", "cu_seqlens", "ids", "targets", "head_order", "row_of_token"):
        assert torch.equal(getattr(a, name), getattr(p, name)), name
    assert HostBatch.of(_batch([5, 3], left=True)["attention_mask"], b["labels"][:2, :5]) is None
    # with the ids too, the packed batch comes from the host in one buffer: the same tensors
    for lengths in ([5, 3, 7], [1, 9], [4], [6, 6, 2, 1]):
        b = _batch(lengths)
        host = HostBatch.of(b["attention_mask"], b["labels"], b["input_ids"])
        a = Packed(b["input_ids"], b["attention_mask"], b["labels"])
        p = Packed(b["input_ids"], b["attention_mask"], b["labels"], host)
        assert host.plan is not None and p.n == a.n and p.n_supervised == a.n_supervised
        for name in ("tok", "pos", "cu_seqlens", "ids", "targets", "head_order", "row_of_token"):
            assert torch.equal(getattr(a, name), getattr(p, name)), (lengths, name)


def test_staging_copies_keep_bytes_dtype_and_shape():
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import staging

    ring = staging(torch.device("cpu"))
    for t in (torch.arange(35, dtype=torch.int64).reshape(5, 7), torch.rand(3, 4) > 0.5,
              torch.randn(6), torch.tensor(3.5)):
        out = ring.tensor_to_device(t, torch.device("cpu"))
        assert out.dtype == t.dtype and out.shape == t.shape and torch.equal(out, t)
    plan = np.arange(10, dtype=np.int64).view(np.uint8)
    assert torch.equal(ring.to_device(plan, torch.device("cpu")), torch.from_numpy(plan))


def test_prepare_inputs_keeps_the_host_facts():
    t, _ = _trainer(_FakeEngine())
    b = _batch([5, 3, 7])
    moved = patch.prepare_inputs(t, dict(b), torch.device("cpu"))
    assert t._qlora_host_batch[0] is moved["input_ids"]
    assert t._qlora_host_batch[1].lengths == [5, 3, 7]


def test_memory_plan_keeps_the_last_layers_and_fits_the_budget():
    from hack_fe30cb28_opus_5_5_ultracode_b200 import memory

    lb, fields = memory.saved_set_bytes(1090, 1536, 12, 2, 128, 8960, 2)
    assert all(off % 256 == 0 for off in fields.values()) and lb >= 1090 * 55_000
    everything = memory.plan_memory(28, lb)
    assert everything.modes == ["keep"] * 28 and everything.ring == 0 and everything.slots == 28
    # a budget for 10 sets: one ring slot for recompute, 9 kept (the last 9 layers)
    p = memory.plan_memory(28, lb, budget_bytes=10 * lb, spill="recompute")
    assert p.modes == ["recompute"] * 19 + ["keep"] * 9 and p.ring == 1 and p.slots == 10
    assert {p.slot(i) for i in range(19)} == {9} and [p.slot(i) for i in range(19, 28)] == list(range(9))
    # offload: two ring slots, alternating between consecutive spilled layers
    q = memory.plan_memory(28, lb, budget_bytes=10 * lb, spill="offload")
    assert q.modes.count("keep") == 8 and q.ring == 2 and q.slots == 10
    assert [q.slot(i) for i in range(4)] == [8, 9, 8, 9]
    assert memory.plan_memory(4, lb, keep_layers=1).modes == ["recompute"] * 3 + ["keep"]
    assert memory.plan_memory(4, lb, budget_bytes=0).modes == ["recompute"] * 4
    with pytest.raises(ValueError):
        memory.plan_memory(4, lb, spill="disk")


def test_step_budget_prediction_and_plan():
    """The predicted step memory (memory.predict_peak_bytes) at the configs[1] shapes: the plans
    differ by their saved-set slots alone (a recompute plan adds its ring slot and the recompute
    scratch), and the budget left for the saved sets after the rest of the step gives a plan
    whose predicted total meets the step budget exactly."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import memory

    n, H, HQ, HKV, D, I, L, V = 1090, 1536, 12, 2, 128, 8960, 28, 151936
    lb, _ = memory.saved_set_bytes(n, H, HQ, HKV, D, I, 2)

    def pred(plan):
        return memory.predict_peak_bytes(L, lb, plan, n, H, V, 2, 0, 1362, 16896, 1 << 24)

    none = pred(memory.MemoryPlan([]))
    assert pred(memory.MemoryPlan(["keep"] * L)) - none == L * lb
    assert pred(memory.MemoryPlan(["recompute"] * L)) - none == lb + n * H * 4
    assert pred(memory.MemoryPlan(["offload"] * L)) - none == 2 * lb
    budget = none + n * H * 4 + 10 * lb
    plan = memory.plan_memory(L, lb, budget - none - n * H * 4, "recompute")
    assert plan.modes.count("keep") == 9 and pred(plan) == budget


def test_gemm_planner_splits_only_long_k_few_tile_products():
    """The GEMM planner (host arithmetic, no GPU needed; 148 SMs assumed without a device) at
    the configs[1] shapes: the long-K products with few output tiles (down projection, gate/up
    and LM-head data gradients at 1,090 tokens) are split in two - the data gradients (MN-major
    B) as 2-SM pair tiles of 256 x 256 (5 x 6 pair tiles, 60 pairs of 148 SMs), whose fp32
    partials need counters + 60 sub-tiles of 128 rows x 2 splits x 128 x 256 floats, the most any
    layout of these shapes asks for; short-K products and large-M products are not split (no
    workspace)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib

    lib = _lib.lib()
    split_two = 2048 + 60 * 2 * 128 * 256 * 4
    n, H, I, V = 1090, 1536, 8960, 151936
    for M, N, K in [(n, H, I), (n, H, 2 * I), (n, H, V)]:
        assert lib.ql_gemm_workspace_bytes(M, N, K) == split_two, (M, N, K)
    for M, N, K in [(n, 2048, H), (n, H, H), (n, I, H), (n, 2 * I, H), (8900, 18944, 3584)]:
        assert lib.ql_gemm_workspace_bytes(M, N, K) == 0, (M, N, K)
    assert lib.ql_gemm_workspace_bytes(0, H, I) == 0


def test_ledger_flushes_accumulated_micro_batches_in_order():
    """Two micro-batches of one optimizer step (gradient accumulation): both are queued on the
    device and written by one flush, in order, with their own training step in the rewind rows;
    a rewind recorder that raises is marked failed and training goes on."""
    t, _ = _trainer(_FakeEngine())
    model = _Model().train()
    first, second = _batch([5, 3, 7]), _batch([4, 6])
    for b in (first, second):
        n_items = int((b["labels"][:, 1:] != -100).sum())
        patch.fused_compute_loss(t, model, dict(b), num_items_in_batch=n_items)
    assert t._metrics["train"]["entropy"] == [] and t._total_train_tokens == 25
    patch.flush_metrics(t)
    assert t._metrics["train"]["entropy"] == [pytest.approx(3.0)] * 2
    assert [r[0] for r in t._soup_rewind_state.rows] == [5, 5]
    assert t._soup_rewind_state.rows[1][2] == [2, 4]
    patch.flush_metrics(t)  # nothing pending: nothing appended
    assert len(t._metrics["train"]["mean_token_accuracy"]) == 2

    class _Broken(_Rewind):
        def on_micro_batch(self, step, row_loss, row_tokens):
            raise RuntimeError("disk full")

    t._soup_rewind_state = _Broken()
    patch.fused_compute_loss(t, model, dict(first), num_items_in_batch=3)
    patch.flush_metrics(t)
    assert t._soup_rewind_state.failed and len(t._metrics["train"]["entropy"]) == 3


def test_packed_partition_without_device_reads_matches_a_stable_sort():
    """The supervised-first order is the stable argsort of 'has no target', for ragged rows, a
    row without any target and an all-prompt batch."""
    for lengths, prompt in (([9, 1, 4, 12], 2), ([3, 3], 5), ([1], 0)):
        b = _batch(lengths, prompt=prompt)
        p = Packed(b["input_ids"], b["attention_mask"], b["labels"])
        want = torch.argsort((p.targets < 0).to(torch.int8), stable=True)
        assert torch.equal(p.head_order, want), lengths
        assert p.n_supervised == int((p.targets >= 0).sum())


def test_auto_plan_offloads_only_what_the_link_can_hide():
    """'auto': with a measured host link and time per layer, every stride-th spilled layer is
    offloaded (counted from the highest spilled one, needed first in the backward) and the others
    recomputed; offloaded layers alternate over two ring slots, recomputed ones share one; with no
    measurement yet everything spilled is recomputed."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import memory

    lb, _ = memory.saved_set_bytes(25000, 1536, 12, 2, 128, 8960, 2)  # 1.4 GB per layer
    # 1.4 GB at 55 GB/s = 25 ms against ~3 ms of forward per layer: every 9th spilled layer
    assert memory.offload_stride(lb, 55.0, 9.25) == 9
    assert memory.offload_stride(lb, None, 9.25) is None
    p = memory.plan_memory(28, lb, budget_bytes=10 * lb, spill="auto", link_gbs=55.0,
                           layer_ms=9.25)
    assert p.modes.count("keep") == 7 and p.ring == 3 and p.slots == 10
    off = [i for i, m in enumerate(p.modes) if m == "offload"]
    assert off == [2, 11, 20] and all(p.modes[i] == "recompute" for i in range(21) if i not in off)
    assert [p.slot(i) for i in off] == [8, 9, 8] and {p.slot(i) for i in (0, 1, 3)} == {7}
    assert memory.plan_memory(28, lb, budget_bytes=10 * lb, spill="auto").summary() == \
        {"keep": 7, "recompute": 21}
    kept = p.with_offload_kept()
    assert kept.summary() == {"keep": 10, "recompute": 18} and kept.slots == 11

"""The whole fused step (embedding, every layer, head; forward + backward) against the CPU oracle
of the reference's step: small random QLoRA Qwen2 models, layers at the 1.5B and 7B widths, and
the benchmarked configs[1] model itself (28 layers, tied V = 151,936, the bench's seeded batch).

Tolerances, fp16: |loss - oracle| <= 1e-3 absolute, every LoRA gradient
within rel-L2 1e-2, the CUDA generator left where PEFT's forward leaves it. bf16 (no reference
step exists in bf16; the oracle rounds to bf16 at the same points): |loss - oracle| <= 5e-3,
LoRA gradients within rel-L2 3e-2 (bf16 keeps 8 significant bits against fp16's 11)."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import step as oracle_step

pytestmark = pytest.mark.gpu
DEV = "cuda"
LOSS_ABS = {torch.float16: 1e-3, torch.bfloat16: 5e-3}
GRAD_REL = {torch.float16: 1e-2, torch.bfloat16: 3e-2}
# fp16 training backpropagates a scaled loss (HF Trainer's GradScaler starts at 2^16) so the
# backward's 16-bit intermediates stay clear of fp16's subnormal range; the gradients are unscaled
# before use. bf16 needs no scale.
LOSS_SCALE = {torch.float16: 65536.0, torch.bfloat16: 1.0}


def _grads(loss, params, dtype):
    """LoRA gradients of the step's loss as fp16 / bf16 training computes them."""
    scale = LOSS_SCALE[dtype]
    grads = torch.autograd.grad(loss, params, grad_outputs=torch.full_like(loss, scale))
    return [g / scale for g in grads]


def _record(name, **values):
    """Appends a test's measured errors to parity_errors.jsonl in the repository's run-output
    folder, when the run created one, so the margins below the bounds are on record."""
    out = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "gpurun_out")
    if os.path.isdir(out):
        with open(os.path.join(out, "parity_errors.jsonl"), "a") as fh:
            fh.write(json.dumps({"test": name, **values}) + "\n")


def _check_step(name, loss, grads, ref, dtype):
    dloss = abs(loss.item() - ref["loss"].item())
    rels = [_rel(g, r_) for g, r_ in zip(grads, ref["grads"])]
    _record(name, dloss=dloss, worst_grad_rel=max(rels), loss=loss.item())
    assert dloss <= LOSS_ABS[dtype], dloss
    assert max(rels) <= GRAD_REL[dtype], (int(np.argmax(rels)), max(rels))


def _batch(lengths, vocab, seed=1, prompt=3):
    g = torch.Generator().manual_seed(seed)
    B, T = len(lengths), max(lengths)
    ids = torch.randint(0, vocab, (B, T), generator=g)
    mask = (torch.arange(T)[None] < torch.tensor(lengths)[:, None]).long()
    ids = torch.where(mask.bool(), ids, 0)
    labels = torch.where(mask.bool(), ids, -100)
    labels[:, :prompt] = -100
    return ids, mask, labels


def _rel(a, b):
    return ((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm().clamp(min=1e-12)).item()


def _run(cfg, lengths, dropout, nested, dtype=torch.float16, seed=1, keep_weights=True,
         **engine_kw):
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import build_qwen2_qlora, lora_parameters

    model = build_qwen2_qlora(cfg, dropout=dropout, device=DEV, seed=seed, nested=nested,
                              embed_dtype=dtype, norm_noise=0.1)
    ids, mask, labels = _batch(lengths, cfg.vocab_size, seed=seed)
    n_items = float((labels[:, 1:] != -100).sum())
    dname = "f16" if dtype == torch.float16 else "bf16"
    W = oracle_step.weights_from_model(model, dname)  # before the engine re-points the bytes
    engine = FusedQwen2(model, dtype=dtype, keep_weights=keep_weights, **engine_kw)
    params = lora_parameters(model)
    gen = torch.cuda.default_generators[torch.cuda.current_device()]
    torch.cuda.manual_seed(5)
    seed0, off0 = gen.initial_seed(), gen.get_offset()
    loss, packed, stats = engine.step(ids.to(DEV), mask.to(DEV), labels.to(DEV), n_items)
    grads = _grads(loss, params, dtype)
    torch.cuda.synchronize()
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    assert ops.device_status() == 0
    state = oracle_step.DropState(seed0, off0, engine.dropout.max_blocks if engine.dropout else 1,
                                  engine.drop_vec)
    ref = oracle_step.step(W, ids, mask, labels, n_items, state)
    return engine, loss, packed, stats, grads, ref, gen


@pytest.mark.parametrize("lengths,dropout,nested", [([17, 60, 33, 5], 0.0, True),
                                                    ([17, 60, 33, 5], 0.1, True),
                                                    ([40, 40], 0.1, False),
                                                    ([4], 0.05, False),
                                                    ([130, 7, 200], 0.05, True)])
def test_fused_step_matches_oracle(lengths, dropout, nested):
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import TINY

    engine, loss, packed, stats, grads, ref, gen = _run(TINY, lengths, dropout, nested)
    _check_step(f"tiny {lengths} p={dropout} nested={nested}", loss, grads, ref, torch.float16)
    order = stats.order.cpu()
    ent = stats.entropy.cpu()
    ref_ent = ref["entropy"][order]
    assert abs(ent.sum().item() - ref_ent.sum().item()) / ref_ent.sum().item() < 1e-3
    assert _rel(stats.tok_loss.cpu(), ref["tok_loss"][order]) < 1e-3
    assert torch.equal(stats.correct.cpu(), ref["correct"][order])
    if dropout > 0:
        assert gen.get_offset() == ref["offset"]


def test_fused_step_full_width_layer_bf16():
    """One decoder layer at the Qwen2.5-1.5B shapes (H 1536, 12 / 2 heads, D 128, I 8960), bf16."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config

    cfg = Qwen2Config(vocab_size=2048, num_hidden_layers=1)
    engine, loss, packed, stats, grads, ref, gen = _run(cfg, [150, 64, 256, 97], 0.05, False,
                                                        dtype=torch.bfloat16)
    _check_step("1.5b-width layer bf16", loss, grads, ref, torch.bfloat16)


@pytest.mark.parametrize("keep_weights", [True, False])
def test_fused_step_full_width_two_layers_fp16(keep_weights):
    """keep_weights=False: the backward dequantises each weight again instead of reading the
    forward's copy."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config

    cfg = Qwen2Config(vocab_size=4096, num_hidden_layers=2)
    engine, loss, packed, stats, grads, ref, gen = _run(cfg, [150, 64, 256, 97], 0.05, True,
                                                        keep_weights=keep_weights)
    _check_step(f"1.5b-width 2 layers fp16 keep_weights={keep_weights}", loss, grads, ref,
                torch.float16)
    assert gen.get_offset() == ref["offset"]


def test_fused_step_qwen25_7b_width_layer_bf16():
    """One decoder layer at the Qwen2.5-7B shapes (H 3584, 28 / 4 heads, D 128, I 18944), bf16:
    the wide-row RMSNorm path, 7-way GQA groups and the 7B GEMM shapes against the oracle."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config

    cfg = Qwen2Config(vocab_size=2048, hidden_size=3584, intermediate_size=18944,
                      num_hidden_layers=1, num_attention_heads=28, num_key_value_heads=4,
                      head_dim=128)
    engine, loss, packed, stats, grads, ref, gen = _run(cfg, [300, 120, 513], 0.05, False,
                                                        dtype=torch.bfloat16)
    _check_step("7b-width layer bf16", loss, grads, ref, torch.bfloat16)


def test_configs1_model_matches_oracle():
    """The benchmarked model itself: Qwen2.5-1.5B (28 layers, tied V = 151,936), NF4 on all
    seven projections, LoRA r16 / alpha 32 / dropout 0.05, fp16, on the first batch bench.py
    times (4 sequences, lognormal lengths, 30 % prompt-masked), against the CPU oracle."""
    import bench
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import (QWEN25_1P5B, build_qwen2_qlora,
                                                             lora_parameters)

    cfg = QWEN25_1P5B
    model = build_qwen2_qlora(cfg, dropout=0.05, device=DEV, seed=0, embed_dtype=torch.float16)
    ids, mask, labels, _ = bench.make_batch(np.random.default_rng(1000), cfg.vocab_size)
    ids, mask, labels = (torch.from_numpy(a) for a in (ids, mask, labels))
    n_items = float((labels[:, 1:] != -100).sum())
    W = oracle_step.weights_from_model(model, "f16")
    engine = FusedQwen2(model, dtype=torch.float16)
    params = lora_parameters(model)
    gen = torch.cuda.default_generators[torch.cuda.current_device()]
    torch.cuda.manual_seed(2024)
    seed0, off0 = gen.initial_seed(), gen.get_offset()
    loss, packed, stats = engine.step(ids.to(DEV), mask.to(DEV), labels.to(DEV), n_items)
    grads = _grads(loss, params, torch.float16)
    torch.cuda.synchronize()
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    assert ops.device_status() == 0
    torch.set_num_threads(os.cpu_count() or 1)
    ref = oracle_step.step(W, ids, mask, labels, n_items,
                           oracle_step.DropState(seed0, off0, engine.dropout.max_blocks,
                                                 engine.drop_vec))
    _check_step("configs[1] 28 layers V=151936 fp16", loss, grads, ref, torch.float16)
    assert gen.get_offset() == ref["offset"]
    order = stats.order.cpu()
    assert _rel(stats.entropy.cpu(), ref["entropy"][order]) < 1e-3


@pytest.fixture
def deterministic_attention():
    """The attention backward in its deterministic form for one test (then the default again)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    ops.attn_set_deterministic(True)
    yield
    ops.attn_set_deterministic(False)


def test_two_steps_are_deterministic(deterministic_attention):
    """Same generator state, same batch: bit-identical loss and LoRA gradients, with the attention
    backward's contributions summed in a fixed order (every other reduction of the step is
    ordered already)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config, build_qwen2_qlora, lora_parameters

    cfg = Qwen2Config(vocab_size=4096, num_hidden_layers=2)
    model = build_qwen2_qlora(cfg, dropout=0.1, device=DEV, seed=3)
    engine = FusedQwen2(model)
    ids, mask, labels = _batch([300, 210, 9, 1100], cfg.vocab_size, seed=4)
    ids, mask, labels = ids.to(DEV), mask.to(DEV), labels.to(DEV)
    params = lora_parameters(model)
    out = []
    for _ in range(2):
        torch.cuda.manual_seed(9)
        loss, _, _ = engine.step(ids, mask, labels, 400.0)
        out.append((loss.detach(), _grads(loss, params, torch.float16)))
    assert torch.equal(out[0][0], out[1][0])
    for a, b in zip(out[0][1], out[1][1]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("keep_layers,spill", [(0, "recompute"), (1, "recompute"), (0, "offload"),
                                               (1, "offload")])
def test_activation_spill_matches_keep_everything(keep_layers, spill, deterministic_attention):
    """Recompute in the backward and offload to pinned host memory give the keep-everything
    step's loss and LoRA gradients bit for bit (same kernels, same dropout draws, the attention
    backward in its deterministic form), as the reference's memory modes do
    (solution/test_kernels.py:429-543)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config, build_qwen2_qlora, lora_parameters

    cfg = Qwen2Config(vocab_size=4096, num_hidden_layers=3)
    ids, mask, labels = _batch([150, 64, 256, 97], cfg.vocab_size, seed=8)
    ids, mask, labels = ids.to(DEV), mask.to(DEV), labels.to(DEV)
    out = []
    for kwargs in ({}, dict(keep_layers=keep_layers, spill=spill)):
        model = build_qwen2_qlora(cfg, dropout=0.1, device=DEV, seed=7)  # the same weights
        params = lora_parameters(model)
        engine = FusedQwen2(model, **kwargs)
        torch.cuda.manual_seed(11)
        loss, _, _ = engine.step(ids, mask, labels, 300.0)
        out.append((loss.detach(), _grads(loss, params, torch.float16), engine.last_plan))
    assert out[1][2].modes.count(spill) == 3 - keep_layers
    assert torch.equal(out[0][0], out[1][0])
    for a, b in zip(out[0][1], out[1][1]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("spill", ["recompute", "offload"])
def test_spilled_layers_match_oracle(spill):
    """Three full-width layers of which the first two spill (recomputed in the backward, or
    offloaded to pinned host memory and fetched back), against the oracle at the same bounds as
    the keep-everything step."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config

    cfg = Qwen2Config(vocab_size=4096, num_hidden_layers=3)
    engine, loss, packed, stats, grads, ref, gen = _run(cfg, [150, 64, 256, 97], 0.05, False,
                                                        spill=spill, keep_layers=1)
    assert engine.last_plan.modes == [spill, spill, "keep"]
    _check_step(f"3 layers, 2 by {spill}", loss, grads, ref, torch.float16)
    assert gen.get_offset() == ref["offset"]


@pytest.mark.parametrize("keep_layers", [None, 1])
def test_streamed_weights_match_resident(keep_layers, deterministic_attention):
    """NF4 base weights in pinned host memory, streamed into two device slots one layer ahead of
    their pass (WeightStream, the reference's solution/engine.py:160-287), give the step with
    resident NF4 bytes its loss and LoRA gradients bit for bit, over two steps, with every layer
    kept or with the first three recomputed in the backward (from the slot their backward uses).
    The layers at each turn of the layer order stay in their slots: the first step copies 2 L - 2
    layers, every later one 2 (L - 2). The bitsandbytes parameters then view the pinned arena."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config, build_qwen2_qlora, lora_parameters

    L = 4
    cfg = Qwen2Config(vocab_size=4096, num_hidden_layers=L)
    ids, mask, labels = _batch([150, 64, 256, 97], cfg.vocab_size, seed=8)
    ids, mask, labels = ids.to(DEV), mask.to(DEV), labels.to(DEV)
    kw = {} if keep_layers is None else dict(keep_layers=keep_layers, spill="recompute")
    runs = []
    for stream in (False, True):
        model = build_qwen2_qlora(cfg, dropout=0.1, device=DEV, seed=7)  # the same weights
        params = lora_parameters(model)
        engine = FusedQwen2(model, keep_weights=False, stream_weights=stream, **kw)
        out, copies = [], []
        for k in range(2):
            torch.cuda.manual_seed(11 + k)
            loss, _, _ = engine.step(ids, mask, labels, 300.0)
            out.append((loss.detach(), _grads(loss, params, torch.float16)))
            if stream:
                copies.append(engine.wstream.copies)
        runs.append((out, engine, copies))
    (resident, _, _), (streamed, engine, copies) = runs
    for (la, ga), (lb, gb) in zip(resident, streamed):
        assert torch.equal(la, lb)
        for a, b in zip(ga, gb):
            assert torch.equal(a, b)
    assert copies == [2 * L - 2, 2 * (L - 2)]
    torch.cuda.synchronize()
    assert engine.wstream.copy_ms() > 0
    for spec in engine.layers:
        for g in (spec.qkv, spec.o, spec.gu, spec.down):
            assert g.packed.device.type == "cpu" and g.packed.is_pinned()
            for p in g.params:
                assert p.data.device.type == "cpu"
                assert p.quant_state.absmax.device.type == "cpu"


def test_streamed_weights_match_oracle():
    """Three full-width layers with streamed NF4 weights (double quantisation: the second-level
    scales stay resident) against the oracle at the keep-everything step's bounds."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config

    cfg = Qwen2Config(vocab_size=4096, num_hidden_layers=3)
    engine, loss, packed, stats, grads, ref, gen = _run(cfg, [150, 64, 256, 97], 0.05, True,
                                                        keep_weights=False, stream_weights=True)
    assert engine.wstream is not None and engine.w16 is None
    _check_step("3 layers, streamed NF4 weights", loss, grads, ref, torch.float16)
    assert gen.get_offset() == ref["offset"]


def test_step_budget_bounds_the_step_memory():
    """step_budget_mib (the reference's predicted-peak planner, solution/engine.py:1630-1707):
    with a budget halfway between the predicted memory of a step that recomputes every layer and
    one that keeps every layer, the plan keeps some layers but not all, and the step's measured
    working memory (the allocator's peak during the step and its backward, above what was
    allocated before it) stays within the prediction for that plan, and so within the budget;
    the prediction is close (within 10 % above the measured peak)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import memory
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config, build_qwen2_qlora, lora_parameters

    L = 6
    cfg = Qwen2Config(vocab_size=4096, num_hidden_layers=L)
    ids, mask, labels = _batch([150, 64, 256, 97], cfg.vocab_size, seed=8)
    ids, mask, labels = ids.to(DEV), mask.to(DEV), labels.to(DEV)
    model = build_qwen2_qlora(cfg, dropout=0.1, device=DEV, seed=7)
    params = lora_parameters(model)
    engine = FusedQwen2(model)
    n, B, T = int(mask.sum()), mask.shape[0], int(mask.sum(1).max())
    keep_all = engine.predict_step_bytes(n, memory.MemoryPlan([memory.KEEP] * L), B, T)
    none = engine.predict_step_bytes(n, memory.MemoryPlan([memory.RECOMPUTE] * L), B, T)
    budget = (keep_all + none) // 2
    engine.step_budget = budget
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    loss, _, _ = engine.step(ids, mask, labels, 300.0)
    _grads(loss, params, torch.float16)
    torch.cuda.synchronize()
    used = torch.cuda.max_memory_allocated() - base
    plan = engine.last_plan
    predicted = engine.predict_step_bytes(n, plan, B, T)
    _record("step budget", used=used, predicted=predicted, budget=budget, plan=plan.summary())
    assert 0 < plan.modes.count(memory.KEEP) < L, plan.summary()
    assert used <= predicted <= budget, (used, predicted, budget)
    assert predicted <= 1.10 * used, (used, predicted)


def test_host_embedding_matches_device_embedding(deterministic_attention):
    """An untied model's input embedding kept in page-locked host memory (host_embedding=True:
    each step's rows gathered over the host link by ql_embed_host) gives the step with the table
    on the device its loss and LoRA gradients bit for bit, and the model's embedding parameter
    then views the pinned table. ql_embed_host gathers exactly the table's rows (the last row
    included) and refuses a table in pageable host memory before launching anything; a tied
    lm_head is refused."""
    import dataclasses

    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib, ops
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import TINY, build_qwen2_qlora, lora_parameters

    cfg = dataclasses.replace(TINY, tie_word_embeddings=False)
    ids, mask, labels = _batch([37, 12, 64], cfg.vocab_size, seed=6)
    ids, mask, labels = ids.to(DEV), mask.to(DEV), labels.to(DEV)
    runs = []
    for host in (False, True):
        model = build_qwen2_qlora(cfg, dropout=0.1, device=DEV, seed=3)  # the same weights
        params = lora_parameters(model)
        engine = FusedQwen2(model, host_embedding=host)
        torch.cuda.manual_seed(4)
        loss, _, _ = engine.step(ids, mask, labels, 90.0)
        runs.append((loss.detach(), _grads(loss, params, torch.float16), engine, model))
    (la, ga, _, _), (lb, gb, engine, model) = runs
    assert torch.equal(la, lb)
    for a, b in zip(ga, gb):
        assert torch.equal(a, b)
    weight = model.get_base_model().model.embed_tokens.weight
    assert weight.device.type == "cpu" and weight.is_pinned()
    table = engine.host_embed
    rows = torch.tensor([0, 5, cfg.vocab_size - 1, 77], device=DEV)
    got = ops.embed(rows, table)
    assert torch.equal(got, table.to(DEV)[rows].float())
    pageable = torch.empty(table.shape, dtype=table.dtype).copy_(table)
    assert not pageable.is_pinned()
    with pytest.raises(_lib.QLError):
        ops.embed(rows, pageable)  # refused before anything is launched
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    with pytest.raises(ValueError):
        FusedQwen2(build_qwen2_qlora(TINY, dropout=0.1, device=DEV, seed=3), host_embedding=True)


def test_kept_weights_follow_the_nf4_storage():
    """The 16-bit weights are dequantised once and reused while the frozen NF4 storage is
    unchanged; an in-place change to a layer's packed bytes (the storage the model's bitsandbytes
    parameters view) refreshes them at the next step."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import TINY

    engine = _run(TINY, [23, 9], 0.0, False)[0]
    spec = engine.layers[0]
    first = engine.w16.clone()
    # a second step with the same weights: nothing is dequantised again, the copy is unchanged
    ids, mask, labels = _batch([23, 9], TINY.vocab_size)
    n_items = float((labels[:, 1:] != -100).sum())
    launches = ops.launch_count()
    engine.step(ids.to(DEV), mask.to(DEV), labels.to(DEV), n_items)[0].backward()
    torch.cuda.synchronize()
    assert torch.equal(engine.w16, first)
    version = engine._w16_version
    # flip bits of layer 0's q projection in place
    storage = spec.qkv.packed
    storage[:64].bitwise_xor_(0x11)
    engine.step(ids.to(DEV), mask.to(DEV), labels.to(DEV), n_items)[0].backward()
    torch.cuda.synchronize()
    assert engine._w16_version != version
    fresh = torch.empty(spec.qkv.shape, device=DEV, dtype=torch.float16)
    spec.qkv.dequant(fresh)
    assert torch.equal(engine.w16[:fresh.numel()].view_as(fresh), fresh)
    assert not torch.equal(engine.w16, first)
    assert ops.launch_count() > launches


def test_pinned_staging_ring_keeps_every_copy():
    """Many more copies than the ring has slots, of growing and shrinking sizes, queued behind
    device work: each device copy holds its own source bytes (a slot is refilled only after the
    copy that last read it)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import PinnedStaging

    dev = torch.device("cuda", 0)
    ring = PinnedStaging()
    busy = torch.randn(4096, 4096, device=dev)
    outs, srcs = [], []
    for i in range(5 * PinnedStaging.SLOTS):
        busy = busy @ busy.t() * 1e-4  # keep the stream busy so copies queue behind it
        src = np.random.default_rng(i).integers(0, 1 << 62, size=1000 + 3000 * (i % 7),
                                                dtype=np.int64)
        srcs.append(src)
        outs.append(ring.to_device(src, dev).view(torch.int64))
    torch.cuda.synchronize()
    for src, out in zip(srcs, outs):
        assert np.array_equal(out.cpu().numpy(), src)

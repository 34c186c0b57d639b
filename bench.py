"""Benchmark of the fused QLoRA training step: train tokens/s of Qwen2.5-1.5B NF4 + LoRA r16 on
1..8 B200 (data parallel), plus peak HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload (per rank): full Qwen2.5-1.5B architecture, random-init weights
(N(0, 0.02), every projection NF4-quantised, tied fp16 embedding / lm_head, V = 151936), LoRA
r16 / alpha 32 / dropout 0.05 on q_proj and v_proj; 4 sequences per step with lognormal lengths
(median 300, clipped to [32, 1024]), token ids uniform in [0, V), labels -100 on the first 30% of
each sequence; one step = fused forward + backward + AdamW (lr 2e-4) on the LoRA weights.
Synthetic data stands in for Soup's Kazakh alpaca set (absent here); each rank draws its own
seeded batches. Timed: exactly K steps between a barrier + synchronize on both sides, CUDA
events, max over ranks; value = real (unpadded) tokens of all ranks / that time.

`e2e` runs the same steps through the drop-in boundary (patch.fused_compute_loss on a trainer
object) from pinned host batches: the host-to-device copy of input_ids / attention_mask / labels
and the loss read back are inside its timed region.

--impl reference times the reference's PyTorch path on the host cores instead (the CPU oracle
restating solution/engine.py in torch fp32): each step one bounded sample (one decoder layer
forward + backward and the head over one sequence of the workload's median length),
extrapolated to the 28-layer model's tokens/s.
"""

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train tokens/s, Qwen2.5-1.5B NF4 QLoRA r16, 1/2/4/8 B200; peak HBM MiB"
WORKLOAD = ("configs[1]: Qwen2.5-1.5B (28 layers, H 1536, 12/2 heads, D 128, I 8960, tied "
            "V 151936), random-init, NF4 on all 7 projections (blocksize 64, fp32 absmax), "
            "fp16 compute, LoRA r16/alpha32/p0.05 on q,v; 4 seqs/rank, lognormal lengths "
            "(median 300, clip [32,1024]), 30% prompt-masked; AdamW lr 2e-4")
SEQS, MEDIAN, LO, HI, PROMPT = 4, 300, 32, 1024, 0.3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--spill", choices=["recompute", "offload"], default=None,
                    help="activation-memory plan: spill all but --keep-layers layers this way "
                         "(default: every layer keeps its activations in HBM)")
    ap.add_argument("--keep-layers", type=int, default=0)
    ap.add_argument("--seqs", type=int, default=SEQS, help="sequences per rank and step")
    ap.add_argument("--median", type=int, default=MEDIAN, help="median sequence length")
    ap.add_argument("--lo", type=int, default=LO)
    ap.add_argument("--hi", type=int, default=HI)
    ap.add_argument("--uniform", default=None, metavar="LO,HI",
                    help="sequence lengths uniform in [LO, HI] instead of lognormal")
    ap.add_argument("--model", choices=["1.5b", "7b"], default="1.5b")
    ap.add_argument("--dtype", choices=["fp16", "bf16"], default="fp16")
    return ap.parse_args()


def make_batch(rng, vocab, seqs=SEQS, median=MEDIAN, lo=LO, hi=HI, uniform=None):
    """Right-padded [B, T] input_ids / attention_mask / labels (HF-style, unshifted)."""
    if uniform is not None:
        lengths = rng.integers(uniform[0], uniform[1] + 1, seqs)
    else:
        lengths = np.clip(np.round(np.exp(rng.normal(math.log(median), 0.6, seqs))), lo,
                          hi).astype(int)
    T = int(lengths.max())
    ids = rng.integers(0, vocab, (seqs, T), dtype=np.int64)
    mask = (np.arange(T)[None, :] < lengths[:, None]).astype(np.int64)
    ids = np.where(mask == 1, ids, 0)
    labels = np.where(mask == 1, ids, -100)
    for r, ln in enumerate(lengths):
        labels[r, :int(round(PROMPT * ln))] = -100
    return ids, mask, labels, int(lengths.sum())


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), \
            "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# CPU: the reference's PyTorch path (oracle), bounded sample
# ---------------------------------------------------------------------------------------------
def cpu_sample(model, seq_len=MEDIAN, layer_index=0):
    """(tokens/s extrapolated to the whole model, seconds, threads, description)."""
    from oracle import step as oracle_step
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import QWEN25_1P5B

    torch.set_num_threads(os.cpu_count() or 1)
    W = oracle_step.weights_from_model_layers(model, [layer_index], "f16")
    L = W["layers"][0]
    g = torch.Generator().manual_seed(7)
    h = torch.randn(seq_len, W["H"], generator=g)
    dh3 = torch.randn(seq_len, W["H"], generator=g)
    pos = torch.arange(seq_len)
    t0 = time.perf_counter()
    oracle_step.layer_forward_backward(W, L, h, [seq_len], pos, dh3)
    t_layer = time.perf_counter() - t0
    ids = torch.randint(0, W["lm"].shape[0], (seq_len,), generator=g)
    t0 = time.perf_counter()
    oracle_step.head_forward_backward(W, h, ids)
    t_head = time.perf_counter() - t0
    layers = QWEN25_1P5B.num_hidden_layers
    total = layers * t_layer + t_head
    desc = (f"one decoder layer fwd+bwd ({t_layer:.2f} s) + head fwd+bwd ({t_head:.2f} s) over "
            f"one {seq_len}-token sequence, fp32 torch on the host, extrapolated to "
            f"{layers} layers")
    return seq_len / total, t_layer + t_head, torch.get_num_threads(), desc


def run_reference(args, rank):
    if rank != 0:
        return
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import QWEN25_1P5B, build_qwen2_qlora

    model = build_qwen2_qlora(QWEN25_1P5B, device="cpu", seed=0, layers_override=1)
    vals, secs, threads, desc = [], [], 1, ""
    for i in range(args.warmup + args.steps):
        v, s, threads, desc = cpu_sample(model)
        if i >= args.warmup:
            vals.append(v)
            secs.append(s)
    value = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.median(secs) * 1000, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp16 rounding points)",
            "data": "synthetic", "config": {"workload": WORKLOAD, "global_batch": SEQS,
                                             "seq_len": "varlen", "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                             "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------------------------
def run_ours(args, rank, world, local):
    import torch.distributed as dist

    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops, patch
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import (QWEN25_1P5B, build_qwen2_qlora,
                                                             lora_parameters)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.barrier(device_ids=[local])
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import QWEN25_7B

    cfg = QWEN25_1P5B if args.model == "1.5b" else QWEN25_7B
    cdt = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    model = build_qwen2_qlora(cfg, dropout=0.05, device=dev, seed=0, embed_dtype=cdt)
    model.train()
    plan_kw = {} if args.spill is None else dict(spill=args.spill, keep_layers=args.keep_layers)
    engine = FusedQwen2(model, dtype=cdt, **plan_kw)
    if world > 1:
        engine.set_data_parallel(None)
    params = lora_parameters(model)
    opt = torch.optim.AdamW(params, lr=2e-4, fused=True)
    rng = np.random.default_rng(1000 + rank)
    uniform = tuple(int(x) for x in args.uniform.split(",")) if args.uniform else None
    host = [make_batch(rng, cfg.vocab_size, args.seqs, args.median, args.lo, args.hi, uniform)
            for _ in range(args.warmup + args.steps)]
    dev_batches = [tuple(torch.from_numpy(a).to(dev) for a in b[:3]) + (b[3],) for b in host]
    denoms = [float((b[2][:, 1:] != -100).sum()) for b in host]

    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import HostBatch

    hosts = [HostBatch.of(torch.from_numpy(b[1]), torch.from_numpy(b[2])) for b in host]

    def train_step(i):
        ids, mask, labels, _ = dev_batches[i]
        loss, _, _ = engine.step(ids, mask, labels, denoms[i], hosts[i])
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    def barrier_sync():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        return float(t.item())

    # The model, the libraries and the batches are set up: move every object made so far out of
    # the cyclic collector's scans, so the steps' short-lived objects do not trigger full scans of
    # them (tens of milliseconds each, which a data-parallel step pays on every rank).
    gc.collect()
    gc.freeze()
    for i in range(args.warmup):
        train_step(i)
    torch.cuda.reset_peak_memory_stats(dev)
    barrier_sync()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    launches0 = ops.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("bench_timed")  # (lets ncu --nvtx-include capture these steps)
    e0.record()
    for i in range(args.warmup, args.warmup + args.steps):
        train_step(i)
    e1.record()
    torch.cuda.nvtx.range_pop()
    barrier_sync()
    launches = ops.launch_count() - launches0
    clk = clocks.stop()
    # Per-operation breakdown and the GEMM roofline: the same K steps again with the library's
    # CUDA-event profiler on (kept out of the timed region: its event pairs cost host time).
    ops.profile_start()
    for i in range(args.warmup, args.warmup + args.steps):
        train_step(i)
    barrier_sync()
    ops.profile_stop()
    prof = ops.profile_read()
    ms = max_over_ranks(e0.elapsed_time(e1))
    peak_mib = torch.cuda.max_memory_allocated(dev) / 2**20  # of the timed plan
    tokens = sum_over_ranks(sum(b[3] for b in host[args.warmup:]))
    mem_line = {"plan": engine.last_plan.summary() if engine.last_plan else None}
    if args.spill is not None:
        # the same steps with every layer kept: the cost of the spill (exposed copy or
        # recompute time) and the host-link traffic it moves
        spill_bytes = engine.last_offload_bytes  # of the last timed step
        keep_layers, engine.keep_layers, engine.spill = engine.keep_layers, None, "recompute"
        barrier_sync()
        e0.record()
        for i in range(args.warmup, args.warmup + args.steps):
            train_step(i)
        e1.record()
        barrier_sync()
        keep_ms = max_over_ranks(e0.elapsed_time(e1))
        engine.keep_layers, engine.spill = keep_layers, args.spill
        mem_line.update(offload_bytes_per_step=spill_bytes,
                        keep_all_ms_per_step=keep_ms / args.steps,
                        spill_ms_per_step=ms / args.steps,
                        exposed_fraction=max(0.0, (ms - keep_ms) / ms))
    value = tokens / (ms / 1000.0)
    gemm_ms = prof.get("gemm", {}).get("ms", 0.0)
    gemm_flops = prof.get("gemm", {}).get("flops", 0.0)
    kernel_ms = {k: round(v["ms"] / args.steps, 4) for k, v in prof.items()}

    # e2e: the drop-in boundary from pinned host batches
    import types

    trainer = types.SimpleNamespace(model=model, args=types.SimpleNamespace(
        average_tokens_across_devices=False, n_gpu=1, fp16=True, bf16=False),
        compute_loss=lambda *a, **k: None, compute_loss_func=None, label_smoother=None,
        model_accepts_loss_kwargs=True, state=types.SimpleNamespace(global_step=0),
        _metrics={"train": {"entropy": [], "mean_token_accuracy": [], "num_tokens": []}},
        _total_train_tokens=0, _soup_rewind_state=None)
    setattr(trainer, patch._ORIGINAL_ATTR, trainer.compute_loss)
    setattr(trainer, patch._INSTALLED_ATTR, engine)
    pinned = [tuple(torch.from_numpy(a).pin_memory() for a in b[:3]) for b in host]

    def e2e_step(i):
        ids, mask, labels = pinned[i]
        inputs = patch.prepare_inputs(trainer, {"input_ids": ids, "attention_mask": mask,
                                                "labels": labels}, dev)
        loss = patch.fused_compute_loss(trainer, model, inputs,
                                        num_items_in_batch=denoms[i])
        loss.backward()
        patch.flush_metrics(trainer)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss.detach().float().item()

    for i in range(min(2, args.warmup)):
        e2e_step(i)
    barrier_sync()
    h2d_total = 0
    e0.record()
    for i in range(args.warmup, args.warmup + args.steps):
        e2e_step(i)
        h2d_total += sum(a.numel() * a.element_size() for a in pinned[i])
    e1.record()
    barrier_sync()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = tokens / (e2e_ms / 1000.0)

    if rank != 0:
        return
    hbm, tf_burst, tf_sust, src = peaks()
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else None
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemm_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as fh:
            traffic = json.load(fh).get("bytes_per_launch")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic (seeded lognormal lengths, uniform token ids, random-init weights)",
        "config": {"workload": WORKLOAD if (args.seqs, args.median, args.lo, args.hi,
                                            args.uniform, args.model, args.dtype) ==
                   (SEQS, MEDIAN, LO, HI, None, "1.5b", "fp16") else
                   f"Qwen2.5-{args.model.upper()} {args.dtype}, {args.seqs} seqs/rank, lengths "
                   + (f"uniform [{args.uniform}]" if args.uniform else
                      f"lognormal (median {args.median}, clip [{args.lo},{args.hi}])"),
                   "global_batch": args.seqs * world, "seq_len": "varlen",
                   "parallelism": f"dp{world}",
                   "l2": "no flush: per-step working set (0.74 GB NF4 weights + GBs of "
                         "activations) is larger than the 126 MB L2",
                   "tokens_per_step_per_rank": tokens / world / args.steps},
        "peak_hbm_mib": peak_mib, "memory": mem_line,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d_total / args.steps,
                "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "roofline": {"kernel": "gemm_tn_kernel (tcgen05, all GEMM launches of the timed steps)",
                     "bound": "tensor", "achieved": achieved, "peak": tf_sust,
                     "unit": "TFLOP/s", "frac": (achieved / tf_sust) if achieved else None,
                     "peak_source": f"{src} bf16 dense, sustained (kernel inside a long step)",
                     "traffic": traffic, "gemm_ms_per_step": gemm_ms / args.steps,
                     "launches": int(prof.get("gemm", {}).get("count", 0))},
        "op_ms_per_step": kernel_ms,
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        v, secs, threads, desc = cpu_sample_from_gpu_model()
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads,
                                "kind": "port", "sample": desc}
    print(json.dumps(line), flush=True)


def cpu_sample_from_gpu_model():
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import QWEN25_1P5B, build_qwen2_qlora

    model = build_qwen2_qlora(QWEN25_1P5B, device="cpu", seed=0, layers_override=1)
    return cpu_sample(model)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the fused QLoRA training step: train tokens/s of Qwen2.5-1.5B NF4 + LoRA r16 on
1..8 B200 (data parallel), plus peak HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload (per rank): full Qwen2.5-1.5B architecture, random-init weights
(N(0, 0.02), every projection NF4-quantised, tied fp16 embedding / lm_head, V = 151936), LoRA
r16 / alpha 32 / dropout 0.05 on q_proj and v_proj; 4 sequences per step with lognormal lengths
(median 300, clipped to [32, 1024]), token ids uniform in [0, V), labels -100 on the first 30% of
each sequence; one step = fused forward + backward + AdamW (lr 2e-4) on the LoRA weights, with
fp16's GradScaler (loss scaled before the backward, gradients unscaled before AdamW) as HF
Trainer runs fp16.
Synthetic data stands in for Soup's Kazakh alpaca set (absent here); each rank draws its own
seeded batches. Timed: exactly K steps between a barrier + synchronize on both sides, CUDA
events, max over ranks; value = real (unpadded) tokens of all ranks / that time.

`e2e` runs the same steps through the drop-in boundary (patch.fused_compute_loss on a trainer
object) from pinned host batches: the host-to-device copy of input_ids / attention_mask / labels,
the ledger's per-step metric read (entropy, accuracy, per-row losses) and the loss read back are
inside its timed region. The loss of step i is read after step i + 1 is launched (as a trainer's
logger reads it), so the host's packing of the next batch overlaps the GPU; the last one is read
before the region closes.

`ops` breaks one step down per operation kind, from the same K steps run again with the library's
event profiler and programmatic dependent launch off (so the per-operation times add up): time
per step, algorithmic bytes (HBM-bound kinds) or FLOPs (GEMMs, attention) and the fraction of the
measured peak. `roofline` is the GEMM class (the largest share of the step).

--impl reference times the reference's PyTorch path on the host cores instead: the CPU oracle
(a torch fp32 restatement of solution/engine.py with its 16-bit rounding points) on the very
batches this arm runs (rank 0's), each step one bounded sample - NF4 dequantisation of one decoder
layer's weights, its forward + backward over the step's whole packed batch, and the head over 256
of its tokens - extrapolated to the 28-layer model and all of the batch's tokens.
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
CPU_SAMPLE_LAYERS = 1  # decoder layers the CPU baseline times per step (then extrapolated)
CPU_HEAD_ROWS = 256    # head rows it times per step (the head's cost is linear in its rows)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--spill", choices=["recompute", "offload", "auto"], default=None,
                    help="activation-memory plan: spill all but --keep-layers layers this way "
                         "(auto: offload only the layers whose copies hide behind compute, "
                         "recompute the rest; default: every layer keeps its activations)")
    ap.add_argument("--keep-layers", type=int, default=None,
                    help="with --spill: keep exactly the last k layers (default 0 without "
                         "--budget-gib)")
    ap.add_argument("--budget-gib", type=float, default=None,
                    help="with --spill: keep as many last layers as fit this many GiB of saved "
                         "activations")
    ap.add_argument("--seqs", type=int, default=SEQS, help="sequences per rank and step")
    ap.add_argument("--median", type=int, default=MEDIAN, help="median sequence length")
    # (--min-len / --max-len under torchrun: its own parser takes --lo for a prefix of --log-dir)
    ap.add_argument("--lo", "--min-len", dest="lo", type=int, default=LO,
                    help="shortest sequence length")
    ap.add_argument("--hi", "--max-len", dest="hi", type=int, default=HI,
                    help="longest sequence length")
    ap.add_argument("--uniform", default=None, metavar="LO,HI",
                    help="sequence lengths uniform in [LO, HI] instead of lognormal")
    ap.add_argument("--stream-weights", action="store_true",
                    help="NF4 base weights in pinned host memory, streamed into two device "
                         "slots one layer ahead (FusedQwen2(stream_weights=True)); the line adds "
                         "the copies' bytes, link rate and exposed time against the same steps "
                         "with the NF4 bytes resident")
    ap.add_argument("--host-embedding", action="store_true",
                    help="the input embedding table in pinned host memory, rows gathered over "
                         "the host link (untied models: --model 7b)")
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


def batches(args, rank, vocab, world=1):
    """The warm-up + timed batches of a rank (both arms draw the same ones). Rank r's sequences
    are drawn from seed 1000 + r; with several ranks, each step's sequences of all ranks are
    dealt back to the ranks token-balanced, args.seqs each (dist.balanced_shards)."""
    uniform = tuple(int(x) for x in args.uniform.split(",")) if args.uniform else None

    def draws(r):
        rng = np.random.default_rng(1000 + r)
        return [make_batch(rng, vocab, args.seqs, args.median, args.lo, args.hi, uniform)
                for _ in range(args.warmup + args.steps)]

    if world == 1:
        return draws(rank)
    from hack_fe30cb28_opus_5_5_ultracode_b200.dist import balanced_shards

    every = [draws(r) for r in range(world)]
    out = []
    for step in range(args.warmup + args.steps):
        rows = []  # (ids, mask, labels) of each sequence of the step, ranks in order
        for r in range(world):
            ids, mask, labels, _ = every[r][step]
            rows += [(ids[i], mask[i], labels[i]) for i in range(ids.shape[0])]
        lengths = [int(m.sum()) for _, m, _ in rows]
        mine = balanced_shards(lengths, world, args.seqs)[rank]
        T = max(lengths[i] for i in mine)
        ids = np.zeros((len(mine), T), dtype=np.int64)
        mask = np.zeros((len(mine), T), dtype=np.int64)
        labels = np.full((len(mine), T), -100, dtype=np.int64)
        for j, i in enumerate(mine):  # right-padded again to this rank's longest sequence
            n = lengths[i]
            ids[j, :n], mask[j, :n], labels[j, :n] = rows[i][0][:n], rows[i][1][:n], rows[i][2][:n]
        out.append((ids, mask, labels, int(sum(lengths[i] for i in mine))))
    return out


def workload_config(args, world):
    """The `config` object of both arms' JSON lines."""
    default = (args.seqs, args.median, args.lo, args.hi, args.uniform, args.model,
               args.dtype) == (SEQS, MEDIAN, LO, HI, None, "1.5b", "fp16")
    name = WORKLOAD if default else (
        f"Qwen2.5-{args.model.upper()} {args.dtype}, {args.seqs} seqs/rank, lengths "
        + (f"uniform [{args.uniform}]" if args.uniform else
           f"lognormal (median {args.median}, clip [{args.lo},{args.hi}])"))
    cfg = {"workload": name, "global_batch": args.seqs * world, "seq_len": "varlen",
           "parallelism": f"dp{world}",
           "l2": "no flush: per-step working set (0.74 GB NF4 weights + GBs of activations) is "
                 "larger than the 126 MB L2"}
    if getattr(args, "host_embedding", False):
        cfg["embedding"] = "input embedding table in pinned host memory, gathered over the link"
    if getattr(args, "stream_weights", False):
        cfg["weights"] = ("NF4 base weights in pinned host memory, streamed into two device "
                          "slots one layer ahead, dequantised per layer pass")
    if world > 1:
        cfg["sharding"] = (f"each step's {args.seqs * world} sequences (rank r's drawn from seed "
                           f"1000 + r) dealt back {args.seqs} per rank, token-balanced "
                           "(longest first to the least-loaded rank)")
    return cfg


def peaks():
    """(HBM GB/s, bf16 TF/s burst, bf16 TF/s sustained, source)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), \
            "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """nvidia-smi clocks / throttle reasons (and the device memory in use) sampled every 200 ms
    during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
              "memory.used")

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
        sm, mx, reasons, used = [], None, set(), []
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
            try:
                used.append(float(parts[9]))
            except (IndexError, ValueError):
                pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "memory_used_mib": max(used) if used else None}


# ---------------------------------------------------------------------------------------------
# CPU: the reference's PyTorch path (oracle), bounded sample of a bench batch
# ---------------------------------------------------------------------------------------------
class CpuSample:
    """Times the CPU oracle on one bench batch: NF4 dequantisation of CPU_SAMPLE_LAYERS decoder
    layers' weights (numpy, inside the timer), their forward + backward over the whole packed
    batch, and the head (final norm, 151,936-way logits, cross-entropy, its backward) over
    CPU_HEAD_ROWS of the batch's tokens, on every host thread; extrapolated to the model's 28
    layers and to all of the batch's head rows."""

    def __init__(self):
        from hack_fe30cb28_opus_5_5_ultracode_b200.model import QWEN25_1P5B, build_qwen2_qlora

        self.cfg = QWEN25_1P5B
        self.model = build_qwen2_qlora(self.cfg, device="cpu", seed=0,
                                       layers_override=CPU_SAMPLE_LAYERS)
        causal = self.model.get_base_model()
        self.embed = causal.model.embed_tokens.weight.detach().float()
        self.norm = causal.model.norm.weight.detach().float()

    def run(self, batch):
        """(tokens/s, seconds of the sample, threads, description)."""
        from oracle import step as oracle_step

        torch.set_num_threads(os.cpu_count() or 1)
        ids, mask, labels, n = batch
        lengths = mask.sum(1).tolist()
        flat = np.flatnonzero(mask.reshape(-1))
        T = mask.shape[1]
        pos = torch.from_numpy(flat % T)
        g = torch.Generator().manual_seed(7)
        h = torch.randn(n, self.cfg.hidden_size, generator=g)
        dh3 = torch.randn(n, self.cfg.hidden_size, generator=g)
        shifted = np.full_like(labels, -100)
        shifted[:, :-1] = labels[:, 1:]
        targets = torch.from_numpy(shifted.reshape(-1)[flat])
        t0 = time.perf_counter()
        W = oracle_step.weights_from_model_layers(self.model, list(range(CPU_SAMPLE_LAYERS)),
                                                  "f16", embed=self.embed, norm=self.norm)
        for L in W["layers"]:
            oracle_step.layer_forward_backward(W, L, h, lengths, pos, dh3)
        t_layers = time.perf_counter() - t0
        rows = min(n, CPU_HEAD_ROWS)
        t0 = time.perf_counter()
        oracle_step.head_forward_backward(W, h[:rows], targets[:rows])
        t_head_sample = time.perf_counter() - t0
        t_head = t_head_sample * n / rows
        layers = self.cfg.num_hidden_layers
        per_layer = t_layers / CPU_SAMPLE_LAYERS
        total = layers * per_layer + t_head
        desc = (f"the bench batch itself ({n} tokens, {len(lengths)} sequences): NF4 dequant + "
                f"fwd+bwd of {CPU_SAMPLE_LAYERS} decoder layer(s) over all tokens "
                f"({per_layer:.2f} s per layer) and the head fwd+bwd over {rows} rows "
                f"({t_head_sample:.2f} s), fp32 torch on the host, extrapolated to {layers} "
                f"layers and {n} head rows")
        return n / total, t_layers + t_head_sample, torch.get_num_threads(), desc


def run_reference(args, rank, world):
    if rank != 0:
        return
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import QWEN25_1P5B

    sample = CpuSample()
    host = batches(args, 0, QWEN25_1P5B.vocab_size, world)
    vals, secs, threads, desc = [], [], 1, ""
    for i in range(args.warmup + args.steps):
        v, s, threads, desc = sample.run(host[i])
        if i >= args.warmup:
            vals.append(v)
            secs.append(s)
    value = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.median(secs) * 1000, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fp16 rounding points)",
            "data": "synthetic (seeded lognormal lengths, uniform token ids, random-init weights)",
            "config": workload_config(args, world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads,
                             "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------------------------
def attention_flops(lengths_per_step, cfg):
    """Algorithmic attention FLOPs per step (forward, backward) over the steps' sequences:
    4 l (l + 1) / 2 HQ D per causal sequence and layer forward, 2.5x that backward."""
    fwd = np.mean([sum(4.0 * L * (L + 1) / 2 for L in lengths) for lengths in lengths_per_step])
    fwd *= cfg.num_attention_heads * cfg.head_dim * cfg.num_hidden_layers
    return fwd, 2.5 * fwd


def op_table(prof, steps, attn, hbm, tf_peak):
    """Per operation kind: ms per step, algorithmic work and the fraction of the peak that bounds
    it (HBM GB/s for the memory-bound kinds, tensor TF/s for GEMMs and attention)."""
    out = {}
    for kind, rec in prof.items():
        ms = rec["ms"] / steps
        row = {"ms_per_step": round(ms, 4), "launches_per_step": rec["count"] / steps}
        flops = rec["flops"] / steps
        if kind == "attn_fwd":
            flops = attn[0]
        elif kind == "attn_bwd":
            flops = attn[1]
        if kind in ("gemm", "attn_fwd", "attn_bwd") and flops and ms:
            tf = flops / (ms / 1e3) / 1e12
            row.update(tflop_per_step=flops / 1e12, achieved_tflops=round(tf, 1),
                       frac_of_bf16_peak=round(tf / tf_peak, 3))
        elif rec["bytes"] and ms:
            gbs = rec["bytes"] / steps / (ms / 1e3) / 1e9
            row.update(gb_per_step=rec["bytes"] / steps / 1e9, achieved_gbs=round(gbs, 1),
                       frac_of_hbm=round(gbs / hbm, 3))
        out[kind] = row
    return out


def run_ours(args, rank, world, local):
    import torch.distributed as dist

    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops, patch
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2, HostBatch
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import (QWEN25_1P5B, QWEN25_7B,
                                                             build_qwen2_qlora, lora_parameters)

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.barrier(device_ids=[local])
    cfg = QWEN25_1P5B if args.model == "1.5b" else QWEN25_7B
    cdt = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    model = build_qwen2_qlora(cfg, dropout=0.05, device=dev, seed=0, embed_dtype=cdt)
    model.train()
    plan_kw = {}
    if args.spill is not None:
        budget = None if args.budget_gib is None else int(args.budget_gib * 1024)
        keep = args.keep_layers if args.keep_layers is not None or budget is not None else 0
        plan_kw = dict(spill=args.spill, keep_layers=keep, activation_budget_mib=budget)
    engine = FusedQwen2(model, dtype=cdt, stream_weights=args.stream_weights,
                        host_embedding=args.host_embedding, **plan_kw)
    if world > 1:
        engine.set_data_parallel(None)
    params = lora_parameters(model)
    opt = torch.optim.AdamW(params, lr=2e-4, fused=True)
    # fp16 mixed precision as HF Trainer runs it: a GradScaler scales the loss before the backward
    # and unscales (and checks) the gradients before the optimizer step; bf16 needs none
    scaler = torch.amp.GradScaler("cuda", enabled=cdt == torch.float16)
    host = batches(args, rank, cfg.vocab_size, world)
    dev_batches = [tuple(torch.from_numpy(a).to(dev) for a in b[:3]) + (b[3],) for b in host]
    denoms = [float((b[2][:, 1:] != -100).sum()) for b in host]
    hosts = [HostBatch.of(torch.from_numpy(b[1]), torch.from_numpy(b[2]), torch.from_numpy(b[0]))
             for b in host]
    timed = range(args.warmup, args.warmup + args.steps)

    def train_step(i):
        ids, mask, labels, _ = dev_batches[i]
        loss, _, _ = engine.step(ids, mask, labels, denoms[i], hosts[i])
        scaler.scale(loss).backward()
        scaler.step(opt)
        scaler.update()
        opt.zero_grad(set_to_none=True)

    def barrier_sync():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def over_ranks(x, op):
        """x combined over the ranks with `op` ("max" or "sum")."""
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
        return float(t.item())

    host_ms = {}

    def timed_steps(step_fn, name=None, finish=None):
        """Device milliseconds of the K timed steps (max over ranks); with a name, also this rank's
        host time to enqueue them (the steps run ahead of the GPU: a host time close to the device
        time means the host, not the GPU, sets the pace). finish: run after the last step, inside
        the timed region (the e2e loop's last host read)."""
        barrier_sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        t0 = time.perf_counter()
        for i in timed:
            step_fn(i)
        if finish is not None:
            finish()
        t1 = time.perf_counter()
        e1.record()
        barrier_sync()
        dev_ms = e0.elapsed_time(e1)
        if name is not None:
            host_ms[name] = ((t1 - t0) * 1e3, dev_ms)
        return over_ranks(dev_ms, "max")

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
    torch.cuda.nvtx.range_push("bench_timed")  # (lets ncu --nvtx-include capture these steps)
    ms = timed_steps(train_step, "timed")
    torch.cuda.nvtx.range_pop()
    launches = ops.launch_count() - launches0
    timed_plan = engine.last_plan  # (the variants below run other plans)
    clk = clocks.stop()
    peak_mib = torch.cuda.max_memory_allocated(dev) / 2**20  # of the timed plan
    tokens = over_ranks(sum(b[3] for b in host[args.warmup:]), "sum")
    # Per-operation breakdown: the same K steps again with the library's event profiler on and
    # programmatic dependent launch off (outside the timed region: event pairs cost host time,
    # and with launches overlapping, per-operation intervals would overlap too).
    ops.set_pdl(False)
    ops.profile_start()
    profiled_ms = timed_steps(train_step)
    ops.profile_stop()
    ops.set_pdl(True)
    prof = ops.profile_read()
    mem_line = {"plan": timed_plan.summary() if timed_plan else None}
    if args.spill is not None:
        from hack_fe30cb28_opus_5_5_ultracode_b200 import memory

        # the spill's costs, each against a variant of the same steps: the copies' exposed time
        # (the plan with its offloaded layers kept instead), the whole spill's cost (every layer
        # kept), and the host-link traffic and its achieved bandwidth (copy-stream events)
        off = engine.last_offload
        torch.cuda.synchronize(dev)
        copy_ms = off.copy_ms() if off is not None else 0.0
        spill_bytes = engine.last_offload_bytes  # of the last timed step
        link_peak = memory.measure_link_gbs(dev)
        variants = {}
        for name, transform, keep in (("offload_kept", memory.MemoryPlan.with_offload_kept,
                                       engine.keep_layers), ("keep_all", None, None)):
            saved = engine.plan_transform, engine.keep_layers, engine.spill
            engine.plan_transform = transform
            if name == "keep_all":
                engine.keep_layers, engine.spill = None, "recompute"
            torch.cuda.reset_peak_memory_stats(dev)
            t = timed_steps(train_step)
            variants[name] = (t, torch.cuda.max_memory_allocated(dev) / 2**20,
                              engine.last_plan.summary())
            engine.plan_transform, engine.keep_layers, engine.spill = saved
        t_kept = variants["offload_kept"][0]
        mem_line.update(
            spill_ms_per_step=ms / args.steps,
            offload_kept_ms_per_step=t_kept / args.steps,
            offload_kept_plan=variants["offload_kept"][2],
            offload_kept_peak_hbm_mib=variants["offload_kept"][1],
            keep_all_ms_per_step=variants["keep_all"][0] / args.steps,
            keep_all_peak_hbm_mib=variants["keep_all"][1],
            exposed_copy_fraction=max(0.0, (ms - t_kept) / ms) if spill_bytes else 0.0,
            offload_bytes_per_step=spill_bytes,
            copy_stream_ms_per_step=copy_ms,
            host_link_gbs=(spill_bytes / (copy_ms / 1e3) / 1e9) if copy_ms else None,
            host_link_peak_gbs=link_peak,
            link_gbs_seen_by_planner=engine.link_gbs, layer_ms_seen_by_planner=engine.layer_ms)
    if args.stream_weights:
        from hack_fe30cb28_opus_5_5_ultracode_b200 import memory

        # the stream's copies (copy-stream events of the last timed step), and the same steps
        # with the NF4 bytes resident and dequantised per layer pass as well (a second engine
        # over the same model: its groups take device copies of the pinned bytes), whose time
        # difference is the copies' exposed time. The second engine runs the streamed engine's
        # last activation plan as it is (no planning of its own from a cold start), so the two
        # differ only in where the NF4 bytes live.
        wst = engine.wstream
        torch.cuda.synchronize(dev)
        copy_ms, moved = wst.copy_ms(), wst.bytes_moved
        streamed = engine
        # the streamed engine's activations (its arena grew to the largest variant above) are
        # released first, to leave the second engine room
        streamed._arena_buf, streamed._saved_cache = None, None
        gc.collect()
        torch.cuda.empty_cache()
        engine = FusedQwen2(model, dtype=cdt, keep_weights=False, **plan_kw)
        same_plan = timed_plan
        engine.plan_transform = lambda _plan: same_plan
        if world > 1:
            engine.set_data_parallel(None)
        for i in range(args.warmup):
            train_step(i)
        t_res = timed_steps(train_step)
        engine = streamed
        mem_line["weight_stream"] = dict(
            layer_mib=wst.layer_bytes / 2**20, host_arena_mib=wst.host.numel() / 2**20,
            device_slots_mib=wst.slots.numel() / 2**20, bytes_per_step=moved,
            copy_stream_ms_per_step=copy_ms,
            host_link_gbs=(moved / (copy_ms / 1e3) / 1e9) if copy_ms else None,
            host_link_peak_gbs=memory.measure_link_gbs(dev),
            resident_ms_per_step=t_res / args.steps, plan=same_plan.summary(),
            exposed_copy_fraction=max(0.0, (ms - t_res) / ms))
    value = tokens / (ms / 1000.0)

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

    # Each step's loss is copied into pinned host memory on the step's stream and read on the host
    # one step later (after the next step's launches), the way a trainer's logger reads it: the
    # host prepares step i + 1 while the GPU still runs step i. The metrics (entropy, accuracy,
    # the per-row losses) are read every step inside the step, by the ledger's flush.
    in_flight = []  # (copy event, pinned loss) not yet read
    losses = []
    slots = [torch.empty((), dtype=torch.float32, pin_memory=True) for _ in range(4)]

    def read_losses(keep):
        while len(in_flight) > keep:
            done, slot = in_flight.pop(0)
            done.synchronize()
            losses.append(float(slot))

    def e2e_step(i):
        ids, mask, labels = pinned[i]
        inputs = patch.prepare_inputs(trainer, {"input_ids": ids, "attention_mask": mask,
                                                "labels": labels}, dev)
        loss = patch.fused_compute_loss(trainer, model, inputs,
                                        num_items_in_batch=denoms[i])
        scaler.scale(loss).backward()
        patch.flush_metrics(trainer)
        scaler.step(opt)
        scaler.update()
        opt.zero_grad(set_to_none=True)
        slot = slots[i % len(slots)]  # (read, two steps back at most, before it is reused)
        slot.copy_(loss.detach().float(), non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        in_flight.append((done, slot))
        read_losses(1)

    for i in range(args.warmup):
        e2e_step(i)
    read_losses(0)
    e2e_ms = timed_steps(e2e_step, "e2e", finish=lambda: read_losses(0))
    if not all(math.isfinite(x) for x in losses):
        raise RuntimeError(f"non-finite e2e losses: {losses}")
    e2e_value = tokens / (e2e_ms / 1000.0)
    h2d = sum(a.numel() * a.element_size() for i in timed for a in pinned[i]) / args.steps
    # the loss (fp32) and the ledger's float64 summary: entropy, correct, supervised, and per row
    # its loss sum and target count
    d2h = 4 + sum(8 * (3 + 2 * pinned[i][0].shape[0]) for i in timed) / args.steps

    # per rank: (host enqueue ms, device ms) per step of the timed and e2e loops
    mine = [host_ms["timed"][0] / args.steps, host_ms["timed"][1] / args.steps,
            host_ms["e2e"][0] / args.steps, host_ms["e2e"][1] / args.steps]
    if world > 1:
        allr = [torch.zeros(4, dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(allr, torch.tensor(mine, dtype=torch.float64, device=dev))
        per_rank = [[round(float(x), 3) for x in t.tolist()] for t in allr]
    else:
        per_rank = [[round(x, 3) for x in mine]]
    if rank != 0:
        return
    hbm, tf_burst, tf_sust, src = peaks()
    # The burst peak applies when the timed steps ran at the maximum SM clock (short steps, no
    # power cap); the sustained one (measured under the power cap) otherwise.
    at_max = clk is not None and clk["sm_max_mhz"] and clk["sm_mhz"] >= 0.95 * clk["sm_max_mhz"] \
        and "sw_power_cap" not in clk["reasons"]
    tf_peak = tf_burst if at_max else tf_sust
    attn = attention_flops([np.asarray(b[1]).sum(1).tolist() for b in host[args.warmup:]], cfg)
    table = op_table(prof, args.steps, attn, hbm, tf_peak)
    gemm = table.get("gemm", {})
    achieved = gemm.get("achieved_tflops")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic (seeded lognormal lengths, uniform token ids, random-init weights)",
        "config": workload_config(args, world),
        "tokens_per_step": tokens / args.steps,
        "peak_hbm_mib": peak_mib, "memory": mem_line,
        # NVML's view: the device memory in use while the timed steps ran (this process's
        # allocator reservations and CUDA context, on a GPU no other process uses)
        "peak_hbm_nvml_mib": clk.get("memory_used_mib") if clk else None,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"kernel": "gemm_tn_kernel + gemm_pair_kernel (tcgen05; every GEMM launch "
                               "of the profiled steps)",
                     "bound": "tensor", "achieved": achieved, "peak": tf_peak,
                     "unit": "TFLOP/s", "frac": (achieved / tf_peak) if achieved else None,
                     "peak_source": f"{src} bf16 dense, "
                                    + ("burst (steps ran at the max SM clock)" if at_max else
                                       "sustained (clocks below max or power-capped)"),
                     "frac_of_burst": (achieved / tf_burst) if achieved else None,
                     "frac_of_sustained": (achieved / tf_sust) if achieved else None,
                     "traffic": None,
                     "traffic_note": "not captured in this run; the ncu DRAM bytes of the "
                                     "GEMMs are in profiles/",
                     "gemm_ms_per_step": gemm.get("ms_per_step"),
                     "launches": int(prof.get("gemm", {}).get("count", 0))},
        "ops": table,
        "ops_note": (f"profiled pass without programmatic dependent launch: "
                     f"{profiled_ms / args.steps:.3f} ms per step, per-op sum "
                     f"{sum(r['ms_per_step'] for r in table.values()):.3f} ms"),
        "clocks": clk,
        "per_rank_ms_per_step": {"fields": ["host_enqueue", "device", "e2e_host", "e2e_device"],
                                 "ranks": per_rank},
    }
    if world == 1 and not args.no_cpu_baseline:
        cpu = CpuSample()
        cpu.run(host[0])  # warm-up: the first call pays for thread pools and allocations
        v, secs, threads, desc = cpu.run(host[args.warmup])
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads,
                                "kind": "port", "sample": desc}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
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

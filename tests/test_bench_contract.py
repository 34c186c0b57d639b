"""CPU: bench.py's reference arm (the reference's algorithm restated on the host cores, as the
driver runs it with --impl reference) prints one JSON line with the contract's keys, the same
metric and unit as the GPU arm, and a cpu_baseline that describes the run."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in line, key
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["value"] > 0
    assert line["metric"].startswith("train tokens/s")
    base = line["cpu_baseline"]
    assert base["kind"] in ("port", "reference") and base["cores"] >= 1 and base["sample"]
    assert base["value"] == line["value"] and base["unit"] == line["unit"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_workload_options_survive_torchrun_parsing():
    """Every workload option reaches bench.py intact through torchrun's own argument parser
    (which takes any prefix of its options, e.g. --lo for --log-dir, as its own)."""
    from torch.distributed.run import get_args_parser

    opts = ["--gpus", "8", "--steps", "10", "--warmup", "3", "--dtype", "bf16", "--seqs", "8",
            "--median", "512", "--min-len", "64", "--max-len", "2048", "--no-cpu-baseline",
            "--stream-weights", "--spill", "auto", "--budget-gib", "40", "--model", "7b",
            "--uniform", "1024,4096", "--impl", "reference"]
    args = get_args_parser().parse_args(["--nnodes=1", "--nproc-per-node", "8", "--master-addr",
                                         "127.0.0.1", "bench.py"] + opts)
    assert args.training_script == "bench.py" and args.training_script_args == opts

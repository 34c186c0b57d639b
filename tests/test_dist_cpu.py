"""CPU, two gloo ranks: the data-parallel gradient reduction of the fused step (GradReducer: any
number of contiguous buckets of the flat gradient buffer, summed and averaged at the end; the
engine uses one bucket, the whole buffer, after the backward) gives every rank the mean of the
ranks' LoRA gradients, and the bench's timing reduction takes the max over ranks."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hack_fe30cb28_opus_5_5_ultracode_b200.dist import GradReducer

        flat = torch.arange(40, dtype=torch.float32) * (rank + 1)
        red = GradReducer()
        for lo in range(0, 40, 10):  # four "layers", last first as in backward
            red.launch(flat[40 - lo - 10:40 - lo])
        red.finish(flat)
        t = torch.tensor([float(rank) * 3.0 + 1.0], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        q.put((rank, flat.tolist(), float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_grad_reducer_averages_over_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=100) for _ in procs]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    expect = [i * 1.5 for i in range(40)]  # mean of i * 1 and i * 2
    for rank, flat, tmax in results:
        assert flat == pytest.approx(expect)
        assert tmax == 4.0


def test_balanced_shards_deal_every_sequence_once_and_even_out_tokens():
    """The bench's data-parallel batches: each step's sequences of all ranks dealt back per_rank
    each, longest first to the least-loaded rank (every sequence exactly once, deterministic),
    evening out the ranks' token counts."""
    import random

    from hack_fe30cb28_opus_5_5_ultracode_b200.dist import balanced_shards

    rng = random.Random(7)
    for ranks, per in ((2, 4), (4, 4), (8, 4), (8, 8), (3, 1)):
        lengths = [int(min(1024, max(32, rng.lognormvariate(5.7, 0.6)))) for _ in range(ranks * per)]
        shards = balanced_shards(lengths, ranks, per)
        assert sorted(i for s in shards for i in s) == list(range(ranks * per))
        assert all(len(s) == per and s == sorted(s) for s in shards)
        assert shards == balanced_shards(lengths, ranks, per)
        loads = [sum(lengths[i] for i in s) for s in shards]
        # no worse than the ranks' own draws, and within one longest sequence of the mean
        own = [sum(lengths[r * per:(r + 1) * per]) for r in range(ranks)]
        assert max(loads) <= max(own)
        assert max(loads) - sum(loads) / ranks <= max(lengths)
    with pytest.raises(ValueError):
        balanced_shards([1, 2, 3], 2, 2)


def test_bench_batches_are_the_dealt_shards():
    """bench.batches with several ranks: the ranks' batches of a step hold every drawn sequence
    once, right-padded, with labels -100 past each length, and rank 0 alone equals its own draws."""
    import sys

    import numpy as np

    sys.argv = ["bench.py", "--steps", "2", "--warmup", "1"]
    import bench

    args = bench.parse()
    world, vocab = 4, 1000
    own = [bench.batches(args, r, vocab) for r in range(world)]
    dealt = [bench.batches(args, r, vocab, world) for r in range(world)]
    for step in range(args.warmup + args.steps):
        drawn = sorted(tuple(ids[i, :m[i].sum()]) for ids, m, _, _ in (o[step] for o in own)
                       for i in range(ids.shape[0]))
        got = []
        for ids, mask, labels, n in (d[step] for d in dealt):
            assert ids.shape == mask.shape == labels.shape and n == int(mask.sum())
            for i in range(ids.shape[0]):
                L = int(mask[i].sum())
                assert mask[i, :L].all() and not mask[i, L:].any()
                assert (labels[i, L:] == -100).all()
                got.append(tuple(ids[i, :L]))
        assert sorted(got) == drawn
    assert all(np.array_equal(a[0], b[0]) for a, b in zip(bench.batches(args, 0, vocab), own[0]))


def _dying_worker(rank, world, port, q):
    """Rank 1 leaves between steps (it exits after the first exchange, as a crashed rank does);
    rank 0 goes on to the next step's gradient exchange, which must end with an error within
    the process group's timeout instead of waiting for good."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    from hack_fe30cb28_opus_5_5_ultracode_b200.dist import GradReducer

    flat = torch.ones(16)
    red = GradReducer()
    red.launch(flat)
    red.finish(flat)  # step 1: both ranks
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the message is written before the process ends
        os._exit(0)  # no destroy_process_group: the peer learns of it from the transport
    t0 = time.monotonic()
    try:
        red.launch(flat)
        red.finish(flat)
        q.put((rank, "no error"))
    except Exception as exc:  # noqa: BLE001 - whatever the backend raises
        q.put((rank, f"error after {time.monotonic() - t0:.1f} s: {type(exc).__name__}"))


@pytest.mark.timeout(120)
def test_a_rank_that_leaves_turns_the_next_exchange_into_an_error():
    """A rank that leaves between steps does not hang the others: their next gradient
    all-reduce raises within the process group's timeout (host-side failure, gloo on CPU)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=100) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error after"), results[0]
    assert float(results[0].split()[2]) < 30.0

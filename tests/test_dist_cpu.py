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

"""Data parallelism of the fused step: each rank packs and runs its own batch on its own GPU
with replicated frozen weights; the only exchange is the LoRA gradients, averaged over the ranks
with NCCL over NVLink (torch.distributed). The reference runs on one GPU only; this is the B200
build's data-parallel layer.

The gradients of the whole model are one flat fp32 buffer (8.7 MB at Qwen2.5-1.5B r16), summed in
one all-reduce after the backward: tens of microseconds over NVLink. Per-layer buckets launched
during the backward (to overlap the exchange with the layers below) measured 12 ms per step
slower on B200 at ~1 k tokens per rank: NCCL's kernels then wait for the slower rank on SMs that
the persistent GEMM grids (one CTA per SM) need.
"""

import torch
import torch.distributed as dist


class GradReducer:
    """Asynchronous bucketed all-reduce of slices of one flat gradient buffer."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.works = []

    def launch(self, bucket):
        """Start summing `bucket` (a contiguous slice of the flat buffer) over the ranks."""
        self.works.append(dist.all_reduce(bucket, op=dist.ReduceOp.SUM, group=self.group,
                                          async_op=True))

    def finish(self, flat):
        """Wait for every launched bucket and turn the sums into means."""
        for w in self.works:
            w.wait()
        self.works = []
        if self.world > 1:
            flat.div_(self.world)
        return flat


def balanced_shards(lengths, ranks, per_rank):
    """Deals a data-parallel step's sequences to the ranks, `per_rank` each, so that the ranks'
    token counts come out as even as a longest-first greedy gets them: each sequence, longest
    first, goes to the least-loaded rank that still has room (ties: the lower rank, then the
    earlier sequence). A rank's step time grows with its token count and every rank waits for
    the slowest in the gradient all-reduce, so an even split is what lets N ranks run N times
    the tokens. Returns one list of sequence indices per rank, each ascending."""
    if len(lengths) != ranks * per_rank:
        raise ValueError(f"{len(lengths)} sequences for {ranks} ranks x {per_rank}")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load, shards = [0] * ranks, [[] for _ in range(ranks)]
    for i in order:
        k = min((r for r in range(ranks) if len(shards[r]) < per_rank),
                key=lambda r: (load[r], r))
        shards[k].append(i)
        load[k] += int(lengths[i])
    return [sorted(s) for s in shards]

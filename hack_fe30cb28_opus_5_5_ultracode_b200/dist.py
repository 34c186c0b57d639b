"""Data parallelism of the fused step: each rank packs and runs its own batch on its own GPU
with replicated frozen weights; the only exchange is the LoRA gradients, averaged over the ranks
with NCCL over NVLink (torch.distributed), one bucket per decoder layer launched as soon as that
layer's backward has written it, so the all-reduce of layer i overlaps the backward of layers
below it. The reference runs on one GPU only; this is the B200 build's data-parallel layer.
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

"""Activation memory of the fused step: where each layer's saved activations live between its
forward and its backward.

The reference (solution/engine.py:290-652, 1630-1707) was written for a 16 GB T4: it plans per
step which layers keep their activations, which recompute them in the backward and which park
inputs, [gate|up] and attention tensors in pinned host memory behind side-stream copies, all
under a fixed cap (solution/patch.py:55-69). On a 180 GB B200 the default plan keeps every
layer (nothing to pay); the same three placements exist here for steps whose activations do not
fit the budget the caller gives:

  keep       the layer's saved set (ql_layer_saved) stays in HBM until its backward;
  recompute  the forward writes the set into a ring slot and drops it; the backward reruns the
             layer's forward from its kept input (bit-identical: same kernels, same dropout
             draws) into the slot, then runs the layer's backward;
  offload    the forward writes the set into a ring slot that a copy stream drains into pinned
             host memory (one cudaMemcpyAsync per layer); the backward copies it back into a
             ring slot one layer ahead, double-buffered against the compute.

Layer inputs (the fp32 residual stream, 6 KB per token per layer at Qwen2.5-1.5B) always stay in
HBM. The last layers are the ones kept: their backward runs first, while the spilled layers'
copies or recomputes come later.
"""

KEEP, RECOMPUTE, OFFLOAD = "keep", "recompute", "offload"


def saved_set_bytes(n, H, HQ, HKV, D, I, elem, align=256):
    """Bytes of one layer's saved set for n tokens (the ql_layer_saved fields, each 256-byte
    aligned), and the per-field offsets, in the order the arena lays them out."""
    sizes = [("rstd1", n * 4), ("yq", n * H * elem), ("yv", n * H * elem),
             ("xq", n * 16 * elem), ("xv", n * 16 * elem), ("q", n * HQ * D * elem),
             ("k", n * HKV * D * elem), ("v", n * HKV * D * elem), ("out", n * HQ * D * elem),
             ("lse", HQ * n * 4), ("h2", n * H * 4), ("rstd2", n * 4), ("gu", n * 2 * I * elem),
             ("keep_q", n * (H // 32) * 4), ("keep_v", n * (H // 32) * 4)]
    fields, off = {}, 0
    for name, b in sizes:
        fields[name] = off
        off = (off + b + align - 1) // align * align
    return off, fields


class MemoryPlan:
    """modes[i] for layer i, and the arena slot each layer's saved set uses."""

    def __init__(self, modes):
        self.modes = list(modes)
        self.kept = [i for i, m in enumerate(self.modes) if m == KEEP]
        spilled = [m for m in self.modes if m != KEEP]
        self.ring = 0 if not spilled else (2 if OFFLOAD in spilled else 1)
        self.slots = len(self.kept) + self.ring
        self._slot = {}
        for k, i in enumerate(self.kept):
            self._slot[i] = k
        r = 0
        for i, m in enumerate(self.modes):
            if m != KEEP:
                self._slot[i] = len(self.kept) + (r % self.ring)
                r += 1

    def slot(self, i):
        return self._slot[i]

    def spilled(self):
        return [i for i, m in enumerate(self.modes) if m != KEEP]

    def summary(self):
        return {m: self.modes.count(m) for m in (KEEP, RECOMPUTE, OFFLOAD) if m in self.modes}


def plan_memory(layers, layer_bytes, budget_bytes=None, spill=RECOMPUTE, keep_layers=None):
    """The step's MemoryPlan. keep_layers: keep exactly the last k layers (a forced plan);
    otherwise keep as many last layers as fit in budget_bytes after the ring slots the spilled
    ones need (None: keep everything)."""
    if spill not in (RECOMPUTE, OFFLOAD):
        raise ValueError(f"spill must be {RECOMPUTE!r} or {OFFLOAD!r}, not {spill!r}")
    if keep_layers is not None:
        k = max(0, min(layers, int(keep_layers)))
    elif budget_bytes is None or layers * layer_bytes <= budget_bytes:
        k = layers
    else:
        ring = 2 if spill == OFFLOAD else 1
        k = max(0, min(layers, (int(budget_bytes) - ring * layer_bytes) // max(layer_bytes, 1)))
    return MemoryPlan([spill] * (layers - k) + [KEEP] * k)

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
AUTO = "auto"  # offload the spilled layers whose copies hide behind compute, recompute the rest


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
    """modes[i] for layer i, and the arena slot each layer's saved set uses: kept layers have
    their own slots; recomputed layers share one ring slot (each is recomputed into it right
    before its backward); offloaded layers alternate between two ring slots (one being refilled
    from host memory while the other is read)."""

    def __init__(self, modes):
        self.modes = list(modes)
        self.kept = [i for i, m in enumerate(self.modes) if m == KEEP]
        self.recompute_ring = 1 if RECOMPUTE in self.modes else 0
        self.offload_ring = 2 if OFFLOAD in self.modes else 0
        self.ring = self.recompute_ring + self.offload_ring
        self.slots = len(self.kept) + self.ring
        self._slot = {}
        for k, i in enumerate(self.kept):
            self._slot[i] = k
        r = 0
        for i, m in enumerate(self.modes):
            if m == RECOMPUTE:
                self._slot[i] = len(self.kept)
            elif m == OFFLOAD:
                self._slot[i] = len(self.kept) + self.recompute_ring + (r % 2)
                r += 1

    def slot(self, i):
        return self._slot[i]

    def spilled(self):
        return [i for i, m in enumerate(self.modes) if m != KEEP]

    def summary(self):
        return {m: self.modes.count(m) for m in (KEEP, RECOMPUTE, OFFLOAD) if m in self.modes}

    def with_offload_kept(self):
        """The same plan with the offloaded layers kept in HBM instead: timed against this plan,
        the difference is the copies' exposed time."""
        return MemoryPlan([KEEP if m == OFFLOAD else m for m in self.modes])


def offload_stride(layer_bytes, link_gbs, layer_ms):
    """Every how many layers one layer's saved set can go to host memory (and come back) without
    the copy showing: its device-to-host copy runs beside the forward of the layers up to the next
    offloaded one, a forward being about a third of a layer's step time layer_ms (the backward,
    twice as long, hides the copy back more easily; the link moves both directions at once).
    None without a measurement."""
    if not link_gbs or not layer_ms or layer_ms <= 0:
        return None
    copy_ms = layer_bytes / (link_gbs * 1e9) * 1e3
    return max(1, int(-(-copy_ms // (layer_ms / 3.0))))


def measure_link_gbs(device, nbytes=64 << 20, reps=4):
    """Host-to-device and device-to-host bandwidth of pinned copies on this device (GB/s, the
    smaller of the two), measured once with CUDA events on a side stream."""
    import torch

    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device=device)
    rates = []
    with torch.cuda.stream(stream):
        for dst, src in ((dev, host), (host, dev)):
            dst.copy_(src, non_blocking=True)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                dst.copy_(src, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            rates.append(reps * nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9)
    return min(rates)


def plan_memory(layers, layer_bytes, budget_bytes=None, spill=RECOMPUTE, keep_layers=None,
                link_gbs=None, layer_ms=None):
    """The step's MemoryPlan.

    keep_layers: keep exactly the last k layers (a forced plan); otherwise keep as many last
    layers as fit in budget_bytes after the ring slots (None: keep everything). The first layers
    spill by `spill`: recompute; offload (all of them); or "auto", which offloads only the layers
    whose copies hide behind compute - every offload_stride-th spilled layer, from the measured
    host-link bandwidth link_gbs and per-layer step time layer_ms - and recomputes the others."""
    if spill not in (RECOMPUTE, OFFLOAD, AUTO):
        raise ValueError(f"spill must be {RECOMPUTE!r}, {OFFLOAD!r} or {AUTO!r}, not {spill!r}")
    if keep_layers is not None:
        k = max(0, min(layers, int(keep_layers)))
    elif budget_bytes is None or layers * layer_bytes <= budget_bytes:
        k = layers
    else:
        ring = {RECOMPUTE: 1, OFFLOAD: 2, AUTO: 3}[spill]
        k = max(0, min(layers, (int(budget_bytes) - ring * layer_bytes) // max(layer_bytes, 1)))
    spilled = layers - k
    if spill == AUTO:
        stride = offload_stride(layer_bytes, link_gbs, layer_ms)
        modes = [RECOMPUTE] * spilled
        if stride is not None:
            # the highest spilled layer is needed first in the backward: count strides from it
            for j in range(spilled - 1, -1, -stride):
                modes[j] = OFFLOAD
        return MemoryPlan(modes + [KEEP] * k)
    return MemoryPlan([spill] * spilled + [KEEP] * k)


def predict_peak_bytes(layers, layer_bytes, plan, n, H, V, elem, fixed_bytes, head_rows,
                       head_width, workspace_bytes):
    """The step's device-memory peak beyond what the model already holds. Held through the
    whole step: the saved-set arena (the plan's slots and the L + 1 fp32 residual slots), the
    head's block buffers (a logits chunk, per row the online state, per supervised row the fp32
    accumulator and chunk product and the 16-bit target row and gradient), the layer workspace,
    the head's input gradient [n, H] fp32 and per-row statistics (rstd, loss, entropy, correct,
    target), the recompute ring's fp32 scratch output, and fixed_bytes (the flat LoRA gradients,
    other per-engine buffers). On top of that, the larger of the head's gathered and normed rows
    (fp32 and 16-bit [n, H], forward only) and the backward's two gradient buffers of each type."""
    h_bytes = (n * H * 4 + 255) // 256 * 256
    arena = plan.slots * layer_bytes + (layers + 1) * h_bytes
    block = head_rows * head_width * elem + head_rows * (4 * 4 + 8 + 4) \
        + head_rows * H * (2 * 4 + 2 * elem)
    held = arena + block + workspace_bytes + n * H * 4 + n * (4 * 4 + 8) + fixed_bytes
    if RECOMPUTE in plan.modes:
        held += n * H * 4
    head_rows_fwd = n * H * (4 + elem)
    backward = 2 * n * H * (4 + elem)
    return held + max(head_rows_fwd, backward)

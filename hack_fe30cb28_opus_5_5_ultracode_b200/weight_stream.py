"""Frozen NF4 base weights kept in pinned host memory and streamed into HBM one layer ahead of
their use (the reference's WeightStream, solution/engine.py:160-287, and its pinned placement,
solution/hostload.py:161-173).

On a 180 GB B200 the NF4 bytes of Qwen2.5-1.5B (0.74 GB) and 7B (3.7 GB) fit next to the
activations, so the engine keeps them resident by default. This stream is for the steps where
they do not: very long packed batches, larger models, several jobs sharing a GPU. Layout:

  host arena  one pinned allocation, layer after layer, each layer the packed bytes and the
              first-level scales (absmax) of its four groups (q|k|v, o, gate|up, down), every
              field 256-byte aligned; the model's bitsandbytes parameters view it, so it is the
              only copy of those bytes;
  two slots   device buffers of one layer each; layer i always uses slot i % 2, so the layer
              descriptors point into their slot once, at set-up.

A pass over layer i (forward, recompute or backward) first waits until slot i % 2 holds layer i,
then queues the copy of the layer it runs next into the other slot on a copy stream (behind the
event that marks the end of that slot's previous pass), so each layer's one cudaMemcpyAsync runs
beside the previous layer's kernels. Because the layer order of a step is 0 .. L-1, L-1 .. 0, the
two layers at each turn (the last two of the forward, the first two of the next step) are still
in their slots: a step copies 2 (L - 2) layers. The second-level scales, code books and offsets of
double quantisation are a few kilobytes per layer and stay resident.

The dequantisation kernels read the slots like any device memory, so a streamed step gives the
resident step's results bit for bit; with the kept 16-bit copy off (keep_weights=False), each
layer pass dequantises its weights from the slot into the layer workspace.

Code outside the fused step (an evaluation, a batch the step does not take) runs the model's own
4-bit layers, which need their bytes on the GPU: restore() copies the arena back into one device
buffer and points the bitsandbytes parameters there; offload(), at the next fused step, points
them at the host arena again and frees that buffer (the reference's restore_weights /
offload_weights, solution/engine.py:1800-1813 and solution/patch.py:280-298).
"""

import torch

GROUPS = ("qkv", "o", "gu", "down")
ALIGN = 256


def _aligned(x):
    return (x + ALIGN - 1) // ALIGN * ALIGN


class WeightStream:
    """layers: the engine's LayerSpecs (their NF4Groups are moved into the host arena);
    descs: their ql_layer_desc structs (the NF4 pointers are set to the slots)."""

    def __init__(self, layers, descs, device):
        self.device = device
        self.L = len(layers)
        # field offsets of one layer, from layer 0 (every layer has the same shapes)
        self.fields = {}
        off = 0
        for name in GROUPS:
            g = getattr(layers[0], name)
            pb = g.packed.numel()
            ab = g.absmax.numel() * g.absmax.element_size()
            self.fields[name] = (off, pb, _aligned(off + pb), ab)
            off = _aligned(_aligned(off + pb) + ab)
        self.layer_bytes = off
        for spec in layers:
            for name in GROUPS:
                g = getattr(spec, name)
                _, pb, _, ab = self.fields[name]
                if g.packed.numel() != pb or g.absmax.numel() * g.absmax.element_size() != ab:
                    raise ValueError(f"layer {spec.index}: {name} differs in size from layer 0")
        # the host arena: each group's bytes moved in, then the group (and the bitsandbytes
        # parameters) re-pointed at them; the device copies are released as each layer is done
        self.layers = layers
        self.absmax_dtype = {name: getattr(layers[0], name).absmax.dtype for name in GROUPS}
        self.host = torch.empty(self.L * self.layer_bytes, dtype=torch.uint8, pin_memory=True)
        for i, spec in enumerate(layers):
            for name in GROUPS:
                g = getattr(spec, name)
                packed, absmax = self._views(self.host, i, name)
                packed.copy_(g.packed.reshape(-1).view(torch.uint8))
                absmax.copy_(g.absmax.reshape(-1))
                g.bind(packed, absmax)
        self.device_copy = None  # the arena's bytes on the GPU while restore()d
        self.slots = torch.empty(2 * self.layer_bytes, device=device, dtype=torch.uint8)
        for i, desc in enumerate(descs):
            base = self.slots.data_ptr() + (i % 2) * self.layer_bytes
            for name in GROUPS:
                po, _, ao, _ = self.fields[name]
                w = getattr(desc, name)  # a view into the descriptor: the writes land in it
                w.packed, w.absmax = base + po, base + ao
        self.stream = torch.cuda.Stream(device=device)
        self.holds = [None, None]   # the layer each slot holds, or is being filled with
        self.ready = [None, None]   # event: the slot's copy has landed
        self.free = [None, None]    # event: the slot's last pass has finished reading it
        self.copies = 0             # layer copies queued since the last reset()
        self.copy_events = []       # (start, end) timing events of those copies

    def _views(self, buf, i, name):
        """Group `name` of layer i in an arena-layout buffer: (packed bytes, absmax)."""
        po, pb, ao, ab = self.fields[name]
        base = i * self.layer_bytes
        return (buf[base + po:base + po + pb],
                buf[base + ao:base + ao + ab].view(self.absmax_dtype[name]))

    def _bind_all(self, buf):
        for i, spec in enumerate(self.layers):
            for name in GROUPS:
                getattr(spec, name).bind(*self._views(buf, i, name))

    def restore(self):
        """The model's 4-bit weights on the GPU again (one copy of the arena), for code that
        runs the model's own layers; the slots and the stream are unchanged."""
        if self.device_copy is None:
            self.device_copy = torch.empty_like(self.host, device=self.device)
            self.device_copy.copy_(self.host)
            self._bind_all(self.device_copy)

    def offload(self):
        """Back to streaming: the weights viewed in the host arena, the device copy freed."""
        if self.device_copy is not None:
            self._bind_all(self.host)
            self.device_copy = None

    def reset(self):
        """Starts a new step's accounting of copies (the slots keep what they hold)."""
        self.copies = 0
        self.copy_events = []

    @property
    def bytes_moved(self):
        return self.copies * self.layer_bytes

    def _copy(self, i):
        s = i % 2
        with torch.cuda.stream(self.stream):
            if self.free[s] is not None:
                self.stream.wait_event(self.free[s])
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(self.stream)
            base = s * self.layer_bytes
            self.slots[base:base + self.layer_bytes].copy_(
                self.host[i * self.layer_bytes:(i + 1) * self.layer_bytes], non_blocking=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record(self.stream)
        self.copy_events.append((t0, t1))
        self.holds[s], self.ready[s] = i, t1
        self.copies += 1

    def use(self, i, nxt=None):
        """Before a pass over layer i on the current stream: makes it wait for layer i's bytes
        (copying them now if no earlier call queued them), then queues the copy of layer nxt,
        the layer the step runs after this one, into the other slot."""
        s = i % 2
        if self.holds[s] != i:
            self._copy(i)
        if self.ready[s] is not None:
            torch.cuda.current_stream().wait_event(self.ready[s])
        if nxt is not None and nxt != i and self.holds[nxt % 2] != nxt:
            self._copy(nxt)

    def done(self, i):
        """After the pass over layer i has been queued: its slot may be refilled once the pass
        has run."""
        ev = torch.cuda.Event()
        ev.record()
        self.free[i % 2] = ev

    def copy_ms(self):
        """Milliseconds the copy stream spent on this step's layer copies (after they ran)."""
        return sum(a.elapsed_time(b) for a, b in self.copy_events)

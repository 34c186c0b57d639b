"""The fused Qwen2 + NF4 + LoRA training step on B200, driving the sm_100a kernels of
libqlora_sm100a.so. Mirrors the reference's FusedQwen2 (solution/engine.py:1568-1922): same
inputs, same outputs (loss, packed batch, per-token statistics), same LoRA gradients through
autograd, same use of the CUDA generator for the LoRA dropout masks.

B200-first differences from the reference (which was built for a 16 GB T4):
  * HBM is plentiful (180 GB), so the default plan keeps every intermediate a layer's backward
    reads instead of recomputing it; NF4 weights stay resident (0.74 GB for 1.5B).
  * every matrix product runs on the tcgen05 GEMM of this library (fp32 accumulation in TMEM);
    each NF4 weight is dequantised once per step, in the forward, into a kept 16-bit copy that
    the backward's data-gradient GEMMs read as an MN-major operand (no second dequantisation,
    no transposed copy; 2.6 GB for 1.5B);
  * LoRA-A products ride in the RMSNorm kernel, LoRA-B products and the LoRA input gradients in
    the RoPE kernels, the residual adds in the GEMM epilogues;
  * attention is this library's varlen causal GQA kernel: k / v are never expanded;
  * the whole model is one autograd Function: forward runs the layers and the head (whose
    gradient is formed in the forward, as the reference's head does), backward runs the layers
    in reverse and hands autograd the LoRA gradients from one flat fp32 buffer, which a
    data-parallel run all-reduces with NCCL.
"""

import ctypes

import numpy as np
import torch
from torch._utils import _unflatten_dense_tensors

from . import _lib, memory, ops

HEAD_CHUNK = 4096          # head rows per block (their per-row statistics and accumulators)
HEAD_L2_BYTES = 40 << 20   # 16-bit logits of one vocabulary chunk of a head block (L2-resident)


# ---------------------------------------------------------------------------------------------
# NF4 weights (solution/engine.py:74-157)
# ---------------------------------------------------------------------------------------------
class NF4Group:
    """The NF4 weights one launch dequantises, read as a single weight of `rows` rows: q, k and
    v; gate and up; or one weight alone. The members share their column count and quantisation
    layout and sit contiguously in device memory in member order (all packed bytes, then all
    first-level scales). With double quantisation each member keeps its own offset, switched at
    the block indices seg1 / seg2, while the second-level scales are concatenated; that is only
    right if every member but the last fills whole second-level blocks, and `split` marks the
    groups where one does not."""

    def __init__(self, params, device):
        states = [p.quant_state for p in params]
        s0 = states[0]
        self.cols = int(s0.shape[1])
        self.rows_each = [int(s.shape[0]) for s in states]
        self.rows = sum(self.rows_each)
        self.nested = bool(s0.nested)
        self.code = s0.code.float().contiguous().to(device)
        if int(s0.blocksize) != 64:
            raise ValueError("NF4 blocksize must be 64")
        for s in states:
            if int(s.shape[1]) != self.cols or bool(s.nested) != self.nested \
                    or int(s.blocksize) != 64 or not torch.equal(s.code.float().to(device), self.code):
                raise ValueError("weights of a group differ in layout")
        blocks = [r * self.cols // 64 for r in self.rows_each]
        # packed bytes and absmax of every member, contiguous
        self.packed = torch.cat([p.data.reshape(-1).view(torch.uint8).to(device) for p in params])
        if self.nested:
            self.bs2 = int(s0.state2.blocksize)
            self.code2 = s0.state2.code.float().contiguous().to(device)
            self.absmax = torch.cat([s.absmax.reshape(-1).to(device) for s in states])
            self.absmax2 = torch.cat([s.state2.absmax.float().reshape(-1).to(device) for s in states])
            self.offsets = torch.stack([torch.as_tensor(s.offset, dtype=torch.float32).reshape(())
                                        .to(device) for s in states])
            self.split = any(b % self.bs2 for b in blocks[:-1])
        else:
            self.bs2 = 1
            self.code2 = self.absmax2 = self.offsets = None
            self.absmax = torch.cat([s.absmax.float().reshape(-1).to(device) for s in states])
            self.split = False
        bounds = []
        for b in blocks[:-1]:
            bounds.append((bounds[-1] if bounds else 0) + b)
        self.seg1, self.seg2 = (bounds + [ops.INT_MAX, ops.INT_MAX])[:2]
        self.blocks = blocks
        self.shape = (self.rows, self.cols)
        self.params = list(params)
        self.bind(self.packed, self.absmax)

    def bind(self, packed, absmax):
        """Makes `packed` / `absmax` (same sizes and dtypes, on the device or in pinned host
        memory) the group's storage, and points the bitsandbytes parameters at them: the model's
        4-bit weights are one copy, wherever the group keeps it."""
        self.packed, self.absmax = packed, absmax
        off_p = off_a = 0
        for p, b in zip(self.params, self.blocks):
            p.data = packed[off_p:off_p + b * 32].view(-1, 1)
            p.quant_state.absmax = absmax[off_a:off_a + b]
            off_p += b * 32
            off_a += b

    def _member(self, i):
        """A view of member i as a single-weight group (for the split nested case)."""
        m = NF4Group.__new__(NF4Group)
        b0 = sum(self.blocks[:i])
        b = self.blocks[i]
        m.cols, m.rows = self.cols, self.rows_each[i]
        m.shape = (m.rows, m.cols)
        m.nested, m.code, m.bs2, m.code2 = self.nested, self.code, self.bs2, self.code2
        m.packed = self.packed[b0 * 32:(b0 + b) * 32]
        m.absmax = self.absmax[b0:b0 + b]
        start2 = sum(-(-x // self.bs2) for x in self.blocks[:i])
        m.absmax2 = self.absmax2[start2:start2 + -(-b // self.bs2)]
        m.offsets = self.offsets[i:i + 1]
        m.seg1 = m.seg2 = ops.INT_MAX
        m.split = False
        return m

    def dequant(self, out, transpose=False):
        """out [rows, cols] (or [cols, rows] with transpose) in out's 16-bit dtype."""
        if not self.split:
            return ops.nf4_dequant(self, out=out, transpose=transpose, dtype=out.dtype)
        r0 = 0
        for i, r in enumerate(self.rows_each):
            part = out[:, r0:r0 + r] if transpose else out[r0:r0 + r]
            if transpose and not part.is_contiguous():
                tmp = torch.empty((self.cols, r), device=out.device, dtype=out.dtype)
                self._member(i).dequant(tmp, transpose=True)
                part.copy_(tmp)
            else:
                self._member(i).dequant(part, transpose=transpose)
            r0 += r
        return out


# ---------------------------------------------------------------------------------------------
# LoRA dropout: the slice of the CUDA generator's Philox stream PEFT's dropout calls consume
# ---------------------------------------------------------------------------------------------
DROPOUT_BLOCK, DROPOUT_UNROLL = 256, 4  # launch constants of aten/src/ATen/native/cuda/Dropout.cu
SELF_CHECK_SEED = 2_718_281_828         # seed of the mask self-check's private RNG fork
SELF_CHECK_SHAPE = (3, 40)              # rows x tokens of the self-check's dropout inputs


def dropout_call(nelem, max_blocks, block=DROPOUT_BLOCK, unroll=DROPOUT_UNROLL):
    """What one aten CUDA dropout call on `nelem` elements takes from the generator, as
    (threads of its grid, Philox offset consumed): the grid is the element count in 256-thread
    blocks, capped at the device's resident blocks; each thread loops over the tensor drawing
    `unroll` values per Philox call (solution/engine.py:787-797 computes the same)."""
    blocks = min(max_blocks, -(-nelem // block))
    passes = -(-nelem // (block * blocks * unroll)) if blocks else 0
    return blocks * block, passes * unroll


class LoraDropoutStream:
    """The Philox draws of PEFT's LoRA dropout calls, reserved from the CUDA generator so this
    library's kernels can regenerate every mask from (seed, counter, threads) and the element's
    index instead of storing it.

    PEFT applies one nn.Dropout per LoRA module in forward order (layer 0 q_proj, layer 0
    v_proj, layer 1 q_proj, ...), each on a contiguous [rows, T, H] input, so every call of a step
    consumes the same offset: `reserve` takes all of a step's calls at once (one read and one
    write of the generator's offset) and hands call k the counter (offset + k * increment) / 4.
    The generator ends exactly where PEFT's own forward leaves it."""

    def __init__(self, device, dtype):
        self.device, self.dtype = device, dtype
        props = torch.cuda.get_device_properties(device)
        self.max_blocks = props.multi_processor_count * (
            props.max_threads_per_multi_processor // DROPOUT_BLOCK)
        index = device.index if device.index is not None else torch.cuda.current_device()
        self.generator = torch.cuda.default_generators[index]
        # aten takes its vectorised path (16-byte loads) on these contiguous inputs
        self.vec = 16 // torch.empty((), dtype=dtype).element_size()
        if self.vec not in (4, 8):
            raise ValueError(f"unsupported LoRA input dtype {dtype}")
        self.verified = None  # outcome of verify(), run once before the first step

    def reserve(self, nelem, calls):
        """(seed as a signed int64, the Philox counter of each of `calls` consecutive dropout calls
        on `nelem` elements, threads of their grid); advances the generator past all of them."""
        if nelem % self.vec:
            raise ValueError(f"{nelem} elements is not a multiple of {self.vec}")
        threads, increment = dropout_call(nelem, self.max_blocks)
        offset = self.generator.get_offset()
        self.generator.set_offset(offset + calls * increment)
        seed = self.generator.initial_seed()
        if seed >> 63:  # the kernels take the 64 seed bits as an int64
            seed -= 1 << 64
        return seed, [(offset + k * increment) // 4 for k in range(calls)], threads

    def verify(self, H, p):
        """Whether this library's masks are the ones torch.nn.functional.dropout draws on this GPU
        and build: two consecutive dropout calls (a layer's q then v input) on a fork of the RNG
        against the RMSNorm kernel's q and v masks from a reservation of the same two calls. The
        training generator is left as it was (torch.random.fork_rng restores it)."""
        rows, tokens = SELF_CHECK_SHAPE
        ones = torch.ones((rows, tokens, H), device=self.device, dtype=self.dtype)
        with torch.random.fork_rng(devices=[self.generator.device]):
            self.generator.manual_seed(SELF_CHECK_SEED)
            seed, (ctr_q, ctr_v), threads = self.reserve(ones.numel(), 2)
            end = self.generator.get_offset()
            self.generator.manual_seed(SELF_CHECK_SEED)
            want_q = torch.nn.functional.dropout(ones, p, training=True) != 0
            want_v = torch.nn.functional.dropout(ones, p, training=True) != 0
            same_end = self.generator.get_offset() == end
        drop = ops.Drop(torch.arange(rows * tokens, device=self.device), seed, ctr_q, ctr_v,
                        threads, p, self.vec)
        out = ops.rms_fwd(torch.ones((rows * tokens, H), device=self.device),
                          torch.ones(H, device=self.device), 1e-6, write_y=False, drop=drop,
                          want_yq=True)
        got_q, got_v = out[2] != 0, out[3] != 0
        return bool(same_end and torch.equal(got_q, want_q.view(rows * tokens, H))
                    and torch.equal(got_v, want_v.view(rows * tokens, H)))


class UnsupportedBatch(ValueError):
    """The fused step does not take this batch; raised before the step changes anything, so the
    caller can run the original code instead (solution/engine.py:700-702)."""


# ---------------------------------------------------------------------------------------------
# per-step packing (solution/engine.py:705-764)
# ---------------------------------------------------------------------------------------------
def _right_padded_lengths(mask):
    """Row lengths of a [rows, T] 0/1 attention mask, or None if some row is not a run of ones
    followed by zeros."""
    m = mask.to(torch.int64)
    valid = bool(((m == 0) | (m == 1)).all()) and bool((m[:, 1:] <= m[:, :-1]).all())
    return m.sum(dim=1).tolist() if valid else None


class HostBatch:
    """What the step needs to know about a batch on the host: each row's length and the number
    of tokens with a target. Computed from the batch while it is still in host memory
    (patch.prepare_inputs), it spares the step the device reads that would otherwise stall the
    host until the previous step's GPU work is done (the reference reads both back,
    solution/engine.py:714, 732)."""

    def __init__(self, lengths, n_supervised, plan=None):
        self.lengths = [int(x) for x in lengths]
        self.n_supervised = int(n_supervised)
        self.plan = plan  # the packed batch's index tensors in one byte array (_host_plan)

    @classmethod
    def of(cls, attention_mask, labels, input_ids=None):
        """From host (CPU) tensors of a right-padded batch; None if it is not right-padded.
        With the token ids as well, the whole packed batch (Packed's index tensors, packed ids,
        targets, head order) is formed here too, so the step moves it to the device in one copy
        instead of a dozen small device operations. (numpy on the host arrays: this runs on the
        step's critical path, before its first launch.)"""
        m = attention_mask.to("cpu").numpy()
        if m.ndim != 2 or not (((m == 0) | (m == 1)).all() and (m[:, 1:] <= m[:, :-1]).all()):
            return None
        lengths = m.sum(axis=1, dtype=np.int64)
        lab = labels.to("cpu").numpy()
        T = lab.shape[1]
        # a token at column t < length - 1 has target labels[row, t + 1]
        has_next = np.arange(T - 1)[None, :] < (lengths[:, None] - 1)
        plan = None
        if input_ids is not None and input_ids.shape == attention_mask.shape:
            plan = _host_plan(lengths, input_ids.to("cpu").numpy(), lab)
        return cls(lengths.tolist(), int(((lab[:, 1:] != -100) & has_next).sum()), plan)


def _index_plan(lengths, T):
    """Host-side int64 indices of the packed tokens, one buffer: [tok | pos | row | cu_seqlens],
    tok = row * T + pos being a token's index in the padded batch."""
    lens = np.asarray(lengths, dtype=np.int64)
    n = int(lens.sum())
    cu = np.zeros(len(lens) + 1, dtype=np.int64)
    np.cumsum(lens, out=cu[1:])
    row = np.repeat(np.arange(len(lens), dtype=np.int64), lens)
    pos = np.arange(n, dtype=np.int64) - cu[:-1][row]
    return np.concatenate([row * T + pos, pos, row, cu]), n


def _host_plan(lengths, ids, lab):
    """Packed's device inputs computed on the host, in one uint8 array: int64 [tok | row | ids |
    targets | head_order] (n each), then int32 [pos (n) | cu_seqlens (B + 1)] - the values the
    device path of Packed forms (the same next-label rule and stable supervised-first order).
    Pageable: the step copies it through its pinned staging ring (PinnedStaging)."""
    B, T = lab.shape
    idx, n = _index_plan(lengths, T)
    tok, pos, row, cu = idx[:n], idx[n:2 * n], idx[2 * n:3 * n], idx[3 * n:]
    nxt = lab.reshape(-1)[np.minimum(tok + 1, max(B * T - 1, 0))] if n else tok
    targets = np.where(pos < T - 1, nxt, -100).astype(np.int64)
    order = np.argsort(targets < 0, kind="stable").astype(np.int64)
    i64 = np.concatenate([tok, row, ids.reshape(-1)[tok].astype(np.int64), targets, order])
    i32 = np.concatenate([pos, cu]).astype(np.int32)
    return np.concatenate([i64.view(np.uint8), i32.view(np.uint8)])


class PinnedStaging:
    """Reusable pinned host buffers for the step's host-to-device copies (its packed batch, and
    the batch tensors a data loader did not pin).
    Pinning host memory (cudaHostAlloc) is slow and may wait for the work already queued on the
    device, so a step that pinned a fresh buffer while the previous step still ran on the GPU
    would stall the host by up to a step; these buffers are pinned once (with headroom, grown
    only for a larger batch), and a slot is refilled only after the copy that last read it has
    finished (its event - long done, a few steps back)."""

    SLOTS = 8

    def __init__(self):
        self.bufs = [None] * self.SLOTS
        self.done = [None] * self.SLOTS
        self.next = 0

    def to_device(self, array, device):
        """A device copy of the bytes of the numpy array `array`, on the current stream."""
        data = np.ascontiguousarray(array).reshape(-1).view(np.uint8)
        if device.type != "cuda":
            return torch.from_numpy(data.copy()).to(device)
        k = self.next
        self.next = (k + 1) % self.SLOTS
        if self.done[k] is not None:
            self.done[k].synchronize()
        buf = self.bufs[k]
        if buf is None or buf.numel() < data.nbytes:
            buf = self.bufs[k] = torch.empty(max(64 << 10, 2 * data.nbytes), dtype=torch.uint8,
                                             pin_memory=True)
        view = buf[:data.nbytes]
        view.numpy()[:] = data
        out = view.to(device, non_blocking=True)
        if self.done[k] is None:
            self.done[k] = torch.cuda.Event()
        self.done[k].record(torch.cuda.current_stream(device))
        return out

    def tensor_to_device(self, t, device):
        """A device copy of the CPU tensor `t` (same dtype and shape) staged through the ring."""
        data = t.contiguous().reshape(-1).view(torch.uint8).numpy()
        return self.to_device(data, device).view(t.dtype).reshape(t.shape)


_STAGING = {}  # device -> PinnedStaging


def staging(device):
    """The process's PinnedStaging ring for copies to `device`."""
    ring = _STAGING.get(device)
    if ring is None:
        ring = _STAGING[device] = PinnedStaging()
    return ring


def _supervised_first(targets):
    """A stable permutation putting the tokens with a target (>= 0) first, without a device
    read: each token's destination is its rank among its own kind, offset by the supervised
    count for the others."""
    n = targets.numel()
    sup = targets >= 0
    seen = torch.cumsum(sup.to(torch.int64), 0)  # supervised tokens up to and including j
    idx = torch.arange(n, device=targets.device)
    dest = torch.where(sup, seen - 1, seen[-1:] + idx - seen) if n else idx
    order = torch.empty_like(idx)
    order.scatter_(0, dest, idx)
    return order, seen


class Packed:
    """One right-padded [rows, T] micro-batch as a single sequence of its real tokens, rows back to
    back (solution/engine.py:705-764 is the reference's): the index tensors the kernels read, the
    next-token targets, and the order the head visits the tokens in (those with a target first,
    so the rows without one can skip the head's backward)."""

    def __init__(self, input_ids, attention_mask, labels, host=None):
        """host: a HostBatch of this batch (then nothing is read back from the device); without
        it the lengths and the supervised count are read back from the device - a host sync, as
        in solution/engine.py:714 - and the right padding is checked there."""
        if input_ids.dim() != 2 or attention_mask.shape != input_ids.shape \
                or labels.shape != input_ids.shape:
            raise UnsupportedBatch("inputs are not [rows, tokens]")
        B, T = input_ids.shape
        if host is None:
            lengths = _right_padded_lengths(attention_mask)
            if lengths is None:
                raise UnsupportedBatch("attention_mask is not right-padded")
        else:
            lengths = list(host.lengths)
            if len(lengths) != B or not all(0 <= x <= T for x in lengths):
                raise UnsupportedBatch("host lengths do not match the batch")
        self.rows, self.T = B, T
        self.lengths = [int(x) for x in lengths]
        self.max_len = max(self.lengths, default=0)
        if host is not None and host.plan is not None:
            self._from_host_plan(host, input_ids.device)
            return
        plan, self.n = _index_plan(self.lengths, T)
        dev = input_ids.device
        staged = staging(dev).to_device(plan, dev).view(torch.int64)
        n = self.n
        self.tok = staged[:n]                        # index in the padded batch (int64)
        self.pos = staged[n:2 * n].to(torch.int32)   # position within its row
        self.row_of_token = staged[2 * n:3 * n]
        self.cu_seqlens = staged[3 * n:].to(torch.int32)
        self.ids = input_ids.reshape(-1).take(self.tok)
        # HF labels are unshifted: a token's target is the label of the next column of its row
        # (-100 past the last column)
        nxt = labels.reshape(-1).take(torch.clamp(self.tok + 1, max=max(B * T - 1, 0)))
        self.targets = torch.where(staged[n:2 * n] < T - 1, nxt, torch.full_like(nxt, -100))
        self.head_order, seen = _supervised_first(self.targets)
        self.n_supervised = host.n_supervised if host is not None \
            else (int(seen[-1]) if n else 0)

    def _from_host_plan(self, host, dev):
        """The packed batch from the host's buffer (HostBatch.plan) in one copy."""
        n = self.n = sum(self.lengths)
        staged = staging(dev).to_device(host.plan, dev)
        i64 = staged[:5 * n * 8].view(torch.int64)
        i32 = staged[5 * n * 8:].view(torch.int32)
        self.tok, self.row_of_token = i64[:n], i64[n:2 * n]
        self.ids, self.targets, self.head_order = i64[2 * n:3 * n], i64[3 * n:4 * n], i64[4 * n:]
        self.pos, self.cu_seqlens = i32[:n], i32[n:]
        self.n_supervised = host.n_supervised


class RopeTable:
    """cos / sin of the model's rotary embedding, first half of head_dim (Qwen2 repeats it)."""

    def __init__(self, rotary, head_dim, device):
        self.rotary, self.half, self.device = rotary, head_dim // 2, device
        self.cos = self.sin = None

    def table(self, length):
        if self.cos is None or self.cos.shape[0] < length:
            size = max(1024, 1 << max(0, (length - 1).bit_length()))
            dummy = torch.zeros(1, device=self.device, dtype=torch.float32)
            pos = torch.arange(size, device=self.device)[None, :]
            with torch.no_grad():
                cos, sin = self.rotary(dummy, pos)
            cos, sin = cos[0].float(), sin[0].float()
            if not (torch.equal(cos[:, :self.half], cos[:, self.half:])
                    and torch.equal(sin[:, :self.half], sin[:, self.half:])):
                raise ValueError("rotary table is not rotate_half style")
            self.cos = cos[:, :self.half].contiguous()
            self.sin = sin[:, :self.half].contiguous()
        return self.cos, self.sin


class HeadStats:
    """Per-token results of the head, in the head's token order (`order`, supervised first):
    `tok_loss` (cross-entropy, 0 without a target), `entropy` of the predicted distribution and
    `correct` (argmax equals the target), the inputs of the logged metrics
    (solution/engine.py:1343-1349 hands back the same four)."""

    __slots__ = ("order", "tok_loss", "entropy", "correct")


# ---------------------------------------------------------------------------------------------
# one decoder layer's weights (solution/engine.py:872-915)
# ---------------------------------------------------------------------------------------------
def _base(module):
    return getattr(module, "base_layer", module)


def _lora_targets(layer):
    found = {}
    for short, module in (("q", layer.self_attn.q_proj), ("k", layer.self_attn.k_proj),
                          ("v", layer.self_attn.v_proj)):
        names = getattr(module, "active_adapters", None)
        if names:
            found[short] = names[0]
    return found


def _lora_dropout(layer, lora_names):
    ps = set()
    for short, name in lora_names.items():
        drop = getattr(layer.self_attn, f"{short}_proj").lora_dropout[name]
        ps.add(float(getattr(drop, "p", 0.0)))
    assert len(ps) <= 1
    return ps.pop() if ps else 0.0


def _lora_input_dtype(layer, lora_names):
    """dtype of the tensor PEFT's LoRA dropout runs on (solution/engine.py:1935-1946): the fp32
    norm output under prepare_model_for_kbit_training, promoted with lora_A's dtype."""
    dtypes = {layer.input_layernorm.weight.dtype}
    for short, name in lora_names.items():
        dtypes.add(getattr(layer.self_attn, f"{short}_proj").lora_A[name].weight.dtype)
    out = dtypes.pop()
    for d in dtypes:
        out = torch.promote_types(out, d)
    return out


class LayerSpec:
    def __init__(self, layer, config, lora_names, index, device, dtype):
        attn, mlp = layer.self_attn, layer.mlp
        self.index = index
        self.H = config.hidden_size
        self.D = getattr(config, "head_dim", None) or self.H // config.num_attention_heads
        self.HQ = config.num_attention_heads
        self.HKV = config.num_key_value_heads
        self.I = config.intermediate_size
        self.C = (self.HQ + 2 * self.HKV) * self.D
        self.eps = float(layer.input_layernorm.variance_epsilon)
        self.ln1 = layer.input_layernorm.weight.detach().float().contiguous()
        self.ln2 = layer.post_attention_layernorm.weight.detach().float().contiguous()
        self.scale = float(attn.scaling)
        w = lambda m: _base(m).weight  # noqa: E731
        self.qkv = NF4Group([w(attn.q_proj), w(attn.k_proj), w(attn.v_proj)], device)
        self.o = NF4Group([w(attn.o_proj)], device)
        self.gu = NF4Group([w(mlp.gate_proj), w(mlp.up_proj)], device)
        self.down = NF4Group([w(mlp.down_proj)], device)
        biases = [_base(getattr(attn, f"{s}_proj")).bias for s in ("q", "k", "v")]
        if any(b is None for b in biases):
            biases = [b if b is not None else torch.zeros(_base(getattr(attn, f"{s}_proj"))
                                                          .weight.quant_state.shape[0],
                                                          device=device)
                      for b, s in zip(biases, ("q", "k", "v"))]
        self.bias_qkv = torch.cat([b.detach().to(dtype) for b in biases]).contiguous()
        self.lora = {}
        for short in ("q", "v"):
            module = getattr(attn, f"{short}_proj")
            if short in lora_names:
                name = lora_names[short]
                self.lora[short] = (module.lora_A[name].weight, module.lora_B[name].weight,
                                    float(module.scaling[name]))
        if set(self.lora) != {"q", "v"}:
            raise ValueError("the fused step needs LoRA on q_proj and v_proj of every layer")
        self.lora_scale = self.lora["q"][2]
        assert self.lora["v"][2] == self.lora_scale

    def lora_params(self):
        return [self.lora["q"][0], self.lora["q"][1], self.lora["v"][0], self.lora["v"][1]]


# ---------------------------------------------------------------------------------------------
# the model
# ---------------------------------------------------------------------------------------------
class FusedQwen2:
    """Holds what the step needs from a PEFT-wrapped, 4-bit Qwen2ForCausalLM."""

    def __init__(self, peft_model, dtype=torch.float16, head_chunk=HEAD_CHUNK, keep_weights=True,
                 spill="recompute", keep_layers=None, activation_budget_mib=None,
                 stream_weights=False, step_budget_mib=None, host_embedding=False):
        """spill / keep_layers / activation_budget_mib: the activation-memory plan of each step
        (memory.plan_memory): by default every layer keeps its saved activations in HBM; with a
        budget (MiB for the saved sets) or a forced keep_layers the first layers spill by
        recompute, by offload to pinned host memory, or "auto": offload only the layers whose
        copies hide behind compute (from the host link's measured bandwidth and the previous
        step's time per layer) and recompute the others.
        stream_weights: move the NF4 base weights into pinned host memory and stream each layer's
        bytes into one of two device slots ahead of its pass (weight_stream.WeightStream); the
        layers then dequantise per pass (no kept 16-bit copy), so HBM holds two layers' NF4
        bytes instead of every layer's NF4 bytes and their 16-bit copy.
        step_budget_mib: a budget for the step's whole working memory instead (the device memory
        a step allocates beyond the model, its optimizer state and the kept weights: saved sets,
        residual slots, backward buffers, head buffers, layer workspace), predicted for each
        step's token count by predict_step_bytes; whatever is left after everything but the
        saved sets goes to the saved sets (the reference's predicted-peak planner,
        solution/engine.py:1630-1707, with a caller's budget in place of its T4 cap).
        host_embedding: keep the input embedding table in page-locked host memory (the model's
        embedding parameter views it) and gather each step's rows from there over the host link
        (the reference's host-resident embedding, solution/offload.py:55-111); only for an untied
        lm_head (a tied head's GEMMs read the table on the device every step); saves the table's
        HBM (1.09 GB for Qwen2.5-7B) for n H 2 bytes of host reads per step."""
        causal = peft_model.get_base_model()
        inner = causal.model
        config = causal.config
        self.dtype = dtype
        self.device = inner.norm.weight.device
        lora_names = _lora_targets(inner.layers[0])
        if "k" in lora_names:
            raise NotImplementedError("LoRA on k_proj")
        self.layers = [LayerSpec(layer, config, lora_names, i, self.device, dtype)
                       for i, layer in enumerate(inner.layers)]
        spec = self.layers[0]
        self.dropout_p = _lora_dropout(inner.layers[0], lora_names)
        self.dropout = LoraDropoutStream(self.device,
                                         _lora_input_dtype(inner.layers[0], lora_names)) \
            if self.dropout_p > 0 else None
        self.drop_vec = self.dropout.vec if self.dropout is not None else 4
        self.norm_w = inner.norm.weight.detach().float().contiguous()
        self.eps = float(inner.norm.variance_epsilon)
        self.embed = inner.embed_tokens.weight.detach().to(dtype).contiguous()
        lm = causal.lm_head.weight.detach()
        self.lm_w = self.embed if lm.data_ptr() == inner.embed_tokens.weight.data_ptr() \
            and lm.dtype == dtype else lm.to(dtype).contiguous()
        self.V = self.lm_w.shape[0]
        self._embed_param = inner.embed_tokens.weight
        self.host_embed = None
        if host_embedding:
            if self.lm_w.data_ptr() == self.embed.data_ptr():
                raise ValueError("host_embedding needs an untied lm_head: a tied head's GEMMs "
                                 "read the embedding table on the device every step")
            self.host_embed = torch.empty(self.embed.shape, dtype=self.embed.dtype,
                                          pin_memory=True)
            self.host_embed.copy_(self.embed)
            self.embed = self.host_embed
            self._embed_to_host()
        self.head = VocabHead(self.lm_w, dtype)
        self.rope = RopeTable(inner.rotary_emb, spec.D, self.device)
        self.head_chunk = head_chunk
        # fp32 LoRA weights (PEFT owns them) and one 16-bit shadow buffer refreshed per step
        self.lora_fp32 = [t for s in self.layers for t in s.lora_params()]
        sizes = [t.numel() for t in self.lora_fp32]
        self.lora_total = sum(sizes)
        self.lora_buf = torch.empty(self.lora_total, device=self.device, dtype=dtype)
        self.lora_views, start = [], 0
        for t, n in zip(self.lora_fp32, sizes):
            self.lora_views.append(self.lora_buf[start:start + n].view(t.shape))
            start += n
        self.offsets = [0]
        for n in sizes:
            self.offsets.append(self.offsets[-1] + n)
        self.process_group = None
        self.data_parallel = False  # LoRA gradients averaged over the ranks (dist.GradReducer)
        self._comm = None           # the all-reduce buffer of the data-parallel gradients
        for spec in self.layers:
            for g in (spec.qkv, spec.o, spec.gu, spec.down):
                if g.split:
                    raise ValueError("double-quantised weights whose absmax2 blocks straddle "
                                     "two members of a group are not supported")
        # the layers' descriptors in one contiguous array (views of it in self.descs), so that
        # the all-layers ABI calls can take them at once
        L = len(self.layers)
        desc_t = _lib.STRUCTS["ql_layer_desc"]
        self.desc_array = (desc_t * L)(*[self._layer_desc(spec) for spec in self.layers])
        self.descs = [self.desc_array[i] for i in range(L)]
        self._step_desc = desc_t()
        self._grad_offsets = (ctypes.c_int64 * L)(*[self.offsets[4 * i] for i in range(L)])
        # the forward's dequantised weights, per layer, read again by the backward
        self.weight_elems = int(_lib.lib().ql_layer_weight_elems(ctypes.byref(self.descs[0])))
        self.wstream = None
        if stream_weights:
            from .weight_stream import WeightStream

            keep_weights = False
            self.wstream = WeightStream(self.layers, self.descs, self.device)
        self.w16 = torch.empty(len(self.layers) * self.weight_elems, device=self.device,
                               dtype=dtype) if keep_weights else None
        self.spill, self.keep_layers = spill, keep_layers
        self.activation_budget = None if activation_budget_mib is None \
            else int(activation_budget_mib) << 20
        self.step_budget = None if step_budget_mib is None else int(step_budget_mib) << 20
        self._host_ring = None     # pinned host memory of offloaded layers (grow-only)
        self._copy_stream = None
        self.link_gbs = None       # host link bandwidth, measured at the first "auto" plan
        self._step_events = None   # (start, end, tokens) of the last step, for the time per layer
        self.layer_ms = None       # the expected time per layer of this step's tokens
        self._layer_ms_per_token = None  # per layer and token, the fastest step seen
        self.last_offload = None   # the last step's _Offload (copy bytes and timing), if any
        self.plan_transform = None  # optional plan -> plan hook (the bench times variants)
        self._scratch_h = None
        self.last_plan = None
        self.last_offload_bytes = 0  # host-link bytes of the last backward's offload plan
        self._workspace = None
        self._arena_buf = None     # grow-only device memory of the saved activations
        self._saved_cache = None   # (key, ql_layer_saved array, residual-slot pointers)
        self._arena_busy = False   # a forward's activations await their backward

    def _layer_desc(self, spec):
        """The step-independent part of a layer's ql_layer_desc (weights, norms, LoRA, dims)."""
        def w(g):
            return _lib.struct("ql_nf4_weight", packed=g.packed.data_ptr(),
                               absmax=g.absmax.data_ptr(), code=g.code.data_ptr(),
                               code2=ops._ptr(g.code2), absmax2=ops._ptr(g.absmax2),
                               offsets=ops._ptr(g.offsets), rows=g.rows, cols=g.cols,
                               seg1=g.seg1, seg2=g.seg2, nested=int(g.nested), bs2=int(g.bs2))

        Aq, Bq, Av, Bv = self.lora_views[4 * spec.index:4 * spec.index + 4]
        return _lib.struct("ql_layer_desc", qkv=w(spec.qkv), o=w(spec.o), gu=w(spec.gu),
                           down=w(spec.down), bias_qkv=spec.bias_qkv.data_ptr(),
                           ln1=spec.ln1.data_ptr(), ln2=spec.ln2.data_ptr(), Aq=Aq.data_ptr(),
                           Bq=Bq.data_ptr(), Av=Av.data_ptr(), Bv=Bv.data_ptr(), eps=spec.eps,
                           scale=spec.scale, lora_scale=spec.lora_scale, H=spec.H, HQ=spec.HQ,
                           HKV=spec.HKV, D=spec.D, I=spec.I, rank=16,
                           dtype=ops.dtype_code(self.dtype))

    def _workspace_for(self, desc):
        need = max(int(_lib.lib().ql_layer_workspace_bytes(ctypes.addressof(desc), 0)),
                   int(_lib.lib().ql_layer_workspace_bytes(ctypes.addressof(desc), 1)))
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = None  # zeroed: its leading GEMM tile counters must start at zero
            self._workspace = torch.zeros(need + need // 4, device=self.device, dtype=torch.uint8)
        return self._workspace

    def restore_weights(self):
        """For code outside the fused step that runs the model's own layers: with streamed
        weights, the NF4 bytes back on the GPU (the next step streams them again), and a
        host-resident embedding table likewise; otherwise nothing to do (the model's parameters
        view the engine's device storage)."""
        if self.wstream is not None:
            self.wstream.restore()
        p = self._embed_param
        if self.host_embed is not None and p.device.type == "cpu":
            p.data = p.data.to(self.device)

    def _embed_to_host(self):
        """The model's embedding parameter views the pinned table (its device copy is freed),
        when the table is kept in the parameter's own dtype."""
        p = self._embed_param
        if p.dtype == self.host_embed.dtype and p.device.type != "cpu":
            p.data = self.host_embed

    def set_data_parallel(self, group=None):
        """Average the LoRA gradients over `group` (None: the default process group) at the end
        of the backward, in one all-reduce of the flat gradient buffer."""
        self.process_group = group
        self.data_parallel = True

    def step(self, input_ids, attention_mask, labels, denom, host=None):
        """One training step's forward: (loss, packed, stats); autograd runs the backward.
        host: an optional HostBatch of this batch (see HostBatch)."""
        packed = Packed(input_ids, attention_mask, labels, host)
        spec = self.layers[0]
        if self.dropout is not None and self.dropout.verified is None:
            self.dropout.verified = self.dropout.verify(spec.H, self.dropout_p)
        if self.dropout is not None and not self.dropout.verified:
            raise UnsupportedBatch("LoRA dropout masks differ from PyTorch's on this GPU "
                                   "(LoraDropoutStream.verify)")
        with torch.no_grad():
            torch._foreach_copy_(self.lora_views, self.lora_fp32)
        if self.wstream is not None:  # (after code outside the step brought the weights back)
            self.wstream.offload()
        if self.host_embed is not None:
            self._embed_to_host()
        stats = HeadStats()
        loss = _FusedStep.apply(self, packed, float(denom), stats, *self.lora_fp32)
        return loss, packed, stats

    # -----------------------------------------------------------------------------------------
    # forward
    # -----------------------------------------------------------------------------------------
    def _drops(self, packed):
        """Each layer's q and v dropout state: PEFT's 2 L dropout calls of this step, reserved
        from the CUDA generator at once (layer i: calls 2 i and 2 i + 1)."""
        L = len(self.layers)
        if self.dropout is None:
            return [ops.Drop(packed.tok, 0, 0, 0, 1, 0.0, 4)] * L
        nelem = packed.rows * packed.T * self.layers[0].H
        seed, ctrs, threads = self.dropout.reserve(nelem, 2 * L)
        return [ops.Drop(packed.tok, seed, ctrs[2 * i], ctrs[2 * i + 1], threads, self.dropout_p,
                         self.drop_vec) for i in range(L)]

    def _forward(self, packed, denom, stats):
        n = packed.n
        spec0 = self.layers[0]
        cos, sin = self.rope.table(max(packed.max_len, 1))
        layer_bytes, _ = memory.saved_set_bytes(n, spec0.H, spec0.HQ, spec0.HKV, spec0.D,
                                                spec0.I, self._esize())
        if self.spill == memory.AUTO:
            if self.link_gbs is None:
                self.link_gbs = memory.measure_link_gbs(self.device)
            ev = self._step_events
            if ev is not None and ev[2] and ev[1].query():  # the previous step has finished
                per_token = ev[0].elapsed_time(ev[1]) / len(self.layers) / ev[2]
                # the fastest step so far sets the estimate: a step the host stalled (the first
                # step's set-up, a host-memory allocation) must not make the next plan offload
                # more layers than the link can hide
                if self._layer_ms_per_token is None or per_token < self._layer_ms_per_token:
                    self._layer_ms_per_token = per_token
            if self._layer_ms_per_token is not None:
                self.layer_ms = self._layer_ms_per_token * n
        budget = self.activation_budget
        if self.step_budget is not None:  # what the rest of the step leaves for the saved sets
            rest = self.predict_step_bytes(n, memory.MemoryPlan([]), packed.rows,
                                           packed.max_len)
            if self.spill != memory.OFFLOAD:
                rest += n * spec0.H * 4  # a recomputed layer's scratch output
            budget = max(0, self.step_budget - rest)
        plan = memory.plan_memory(len(self.layers), layer_bytes, budget,
                                  self.spill, self.keep_layers, self.link_gbs, self.layer_ms)
        if self.plan_transform is not None:
            plan = self.plan_transform(plan)
        self.last_plan = plan
        if self.spill == memory.AUTO:
            self._step_events = (torch.cuda.Event(enable_timing=True),
                                 torch.cuda.Event(enable_timing=True), n)
            self._step_events[0].record()
        arena = _SavedArena(n, spec0, len(self.layers), self.dtype, self.device,
                            None if self._arena_busy else self._arena_buf, plan)
        offload = _Offload(self, arena, plan) if memory.OFFLOAD in plan.modes and n else None
        if not self._arena_busy:
            self._arena_buf = arena.buf
            self._arena_busy = True
            arena.owned = True
        h = arena.h(0)
        if n:
            ops.embed(packed.ids, self.embed, out=h)
            if self.w16 is not None:  # the 16-bit weights of every layer, few launches
                self._dequant_all()
        L = len(self.layers)
        drops = self._drops(packed)
        self._set_all_steps(packed, drops, cos, sin)
        saved_arr, h_out = self._saved_structs(arena, plan)
        wst = self.wstream
        if wst is not None:
            wst.reset()
        if n and all(m == memory.KEEP for m in plan.modes) and wst is None:
            # every layer keeps its saved set: the whole forward in one call
            ws = self._workspace_for(self.descs[0])
            _lib.call("ql_layers_forward", ctypes.addressof(self.desc_array),
                      ctypes.addressof(saved_arr), L, ctypes.addressof(h_out), ws.data_ptr(),
                      ws.numel(), ops.stream_ptr())
        elif n:
            for i, desc in enumerate(self.descs):
                if offload is not None:
                    offload.before_forward(i)
                if wst is not None:  # layer i's NF4 bytes in its slot, layer i + 1's on the way
                    wst.use(i, i + 1 if i + 1 < L else None)
                ws = self._workspace_for(desc)
                _lib.call("ql_layer_forward", ctypes.addressof(desc),
                          ctypes.addressof(saved_arr[i]), arena.h(i + 1).data_ptr(),
                          ws.data_ptr(), ws.numel(), ops.stream_ptr())
                if wst is not None:
                    wst.done(i)
                if offload is not None:
                    offload.after_forward(i)
        saved = (saved_arr, drops)
        h = arena.h(len(self.layers))
        dhp, loss = self._head(h, packed, denom, stats) if n else (None, None)
        if loss is None:
            loss = torch.zeros((), device=self.device)
        return loss, (arena, saved, offload), dhp

    def predict_step_bytes(self, n, plan, seqs=None, max_len=None):
        """Predicted device memory a step of n tokens (seqs sequences, the longest max_len
        tokens; by default one sequence of n) allocates under `plan` beyond what the model
        already holds (memory.predict_peak_bytes with this engine's shapes, head block and layer
        workspace)."""
        spec = self.layers[0]
        e = self._esize()
        layer_bytes, _ = memory.saved_set_bytes(n, spec.H, spec.HQ, spec.HKV, spec.D, spec.I, e)
        rows = min(n, self.head_chunk)
        width = self.head.chunk_width(rows) if rows else 0
        # the layer workspace for this step's sizes, from a copy of a layer's descriptor
        desc = _lib.STRUCTS["ql_layer_desc"].from_buffer_copy(self.descs[0])
        desc.n, desc.B = n, seqs if seqs is not None else 1
        desc.max_len = max_len if max_len is not None else n
        ws = max(int(_lib.lib().ql_layer_workspace_bytes(ctypes.addressof(desc), b))
                 for b in (0, 1))
        # the head's block buffers and the workspace are allocated with a quarter of headroom;
        # fixed: the flat LoRA gradients and one more set (a caller's unscaled or accumulated
        # copies), and an allowance for the packed batch's index tensors, the RoPE tables and
        # other small temporaries
        fixed = 2 * self.lora_total * 4 + n * 64 + (8 << 20)
        return memory.predict_peak_bytes(len(self.layers), layer_bytes, plan, n, spec.H, self.V,
                                         e, fixed, rows + rows // 4, width, ws + ws // 4)

    def _saved_structs(self, arena, plan):
        """Every layer's ql_layer_saved (device addresses in the arena) and the residual slots
        the layers write. They depend only on the arena's address, the token count and the plan,
        so the arrays are rebuilt only when one of those changes (a new array is made then: the
        previous one may still be held by a step whose backward has not run)."""
        L = len(self.layers)
        w16 = self.w16.data_ptr() if self.w16 is not None else 0
        key = (arena.base, arena.n, tuple(plan.modes), w16)
        if self._saved_cache is None or self._saved_cache[0] != key:
            # every address is base + offsets: filled as one [L, 18] array of 8-byte words (the
            # struct's 17 pointers, then w16_ready and its padding) and copied in at once, since
            # the token count - and with it the layout - changes from step to step
            st = _lib.STRUCTS["ql_layer_saved"]
            names = [f for f, _ in st._fields_]
            if ctypes.sizeof(st) != 18 * 8 or names[-1] != "w16_ready" or names[0] != "h":
                raise RuntimeError("ql_layer_saved layout changed")
            slots = np.array([plan.slot(i) for i in range(L)], dtype=np.uint64)
            base = np.uint64(arena.base) + slots * np.uint64(arena.layer_bytes)
            words = np.zeros((L, 18), dtype=np.uint64)
            h0 = arena.base + arena.slots * arena.layer_bytes
            words[:, 0] = h0 + np.arange(L, dtype=np.uint64) * np.uint64(arena.h_bytes)
            for j, name in enumerate(names[1:16], start=1):
                words[:, j] = base + np.uint64(arena.fields[name])
            if w16:
                words[:, 16] = np.uint64(w16) + np.arange(L, dtype=np.uint64) * np.uint64(
                    self.weight_elems * self._esize())
                words[:, 17] = 1  # w16_ready (little-endian int32 in the low half)
            saved_arr = (st * L)()
            ctypes.memmove(saved_arr, words.ctypes.data, words.nbytes)
            h_out = (ctypes.c_void_p * L)(*(words[:, 0] + np.uint64(arena.h_bytes)).tolist())
            self._saved_cache = (key, saved_arr, h_out)
        return self._saved_cache[1], self._saved_cache[2]

    def _nf4_version(self):
        """Sum of the version counters of every NF4 tensor the kept weights come from (packed
        bytes, scales): it grows whenever one of them is written in place."""
        if getattr(self, "_nf4_tensors", None) is None:
            ts = []
            for spec in self.layers:
                for g in (spec.qkv, spec.o, spec.gu, spec.down):
                    ts += [g.packed, g.absmax] + ([g.absmax2, g.offsets] if g.nested else [])
            self._nf4_tensors = ts
        return sum(t._version for t in self._nf4_tensors)

    def _dequant_all(self):
        """Every layer's four NF4 groups into the kept 16-bit weights ([qkv | o | gate_up |
        down] per layer, as the layer kernels lay them out) with ql_nf4_dequant_batch. The base
        weights are frozen, so the kept copy is refreshed only when the NF4 storage has changed
        since the last dequantisation (its version counters) - once, for training as usual:
        every later step reads the same 16-bit weights a fresh dequantisation would write."""
        version = self._nf4_version()
        if getattr(self, "_w16_version", None) == version:
            return
        if getattr(self, "_dq_args", None) is None:
            spec = self.layers[0]
            C = (spec.HQ + 2 * spec.HKV) * spec.D
            offs = [0, C * spec.H, C * spec.H + spec.H * spec.HQ * spec.D,
                    C * spec.H + spec.H * spec.HQ * spec.D + 2 * spec.I * spec.H]
            e = self._esize()
            groups, outs = [], []
            for i, desc in enumerate(self.descs):
                base = self.w16.data_ptr() + i * self.weight_elems * e
                for g, off in zip((desc.qkv, desc.o, desc.gu, desc.down), offs):
                    groups.append(g)
                    outs.append(base + off * e)
            arr = (_lib.STRUCTS["ql_nf4_weight"] * len(groups))(*groups)
            ptrs = (ctypes.c_void_p * len(outs))(*outs)
            self._dq_args = (arr, ptrs, len(groups))
        arr, ptrs, count = self._dq_args
        _lib.call("ql_nf4_dequant_batch", ctypes.addressof(arr), ctypes.addressof(ptrs), count,
                  ops.dtype_code(self.dtype), ops.stream_ptr())
        self._w16_version = version

    def _esize(self):
        return torch.empty((), dtype=self.dtype).element_size()

    def _recompute(self, i, desc, sv, arena):
        """Reruns layer i's forward from its kept input into its (ring) saved set."""
        n, H = arena.n, arena.H
        if self._scratch_h is None or self._scratch_h.numel() < n * H:
            self._scratch_h = torch.empty(n * H, device=self.device, dtype=torch.float32)
        ws = self._workspace_for(desc)
        _lib.call("ql_layer_forward", ctypes.addressof(desc), ctypes.addressof(sv),
                  self._scratch_h.data_ptr(), ws.data_ptr(), ws.numel(), ops.stream_ptr())

    def _set_all_steps(self, packed, drops, cos, sin):
        """The step-dependent fields of every layer's descriptor (ql_layers_set_step): the
        shared ones through one template descriptor, each layer's dropout counters."""
        L = len(self.layers)
        self._set_step(self._step_desc, packed, drops[0], cos, sin)
        ctr_q = (ctypes.c_int64 * L)(*[d.ctr_q for d in drops])
        ctr_v = (ctypes.c_int64 * L)(*[d.ctr_v for d in drops])
        _lib.call("ql_layers_set_step", ctypes.addressof(self.desc_array), L,
                  ctypes.addressof(self._step_desc), ctypes.addressof(ctr_q),
                  ctypes.addressof(ctr_v))

    def _set_step(self, desc, packed, drop, cos, sin):
        """The step-dependent fields of a layer's descriptor."""
        desc.cos, desc.sin = cos.data_ptr(), sin.data_ptr()
        desc.pos, desc.cu_seqlens = packed.pos.data_ptr(), packed.cu_seqlens.data_ptr()
        desc.tok = packed.tok.data_ptr()
        desc.n, desc.B, desc.max_len = packed.n, packed.rows, packed.max_len
        f = drop.fields()
        desc.seed, desc.ctr_q, desc.ctr_v, desc.threads = (f["seed"], f["ctr_q"], f["ctr_v"],
                                                           f["threads"])
        desc.p_keep, desc.keep_scale, desc.vec = f["p_keep"], f["keep_scale"], f["vec"]
        desc.drop_q, desc.drop_v = f["drop_q"], f["drop_v"]

    def _head(self, h, packed, denom, stats):
        """Final norm, lm_head, cross-entropy and the logged metrics, with the gradient w.r.t.
        the final hidden state formed in the same pass (solution/engine.py:1352-1400, and the
        vocabulary-piece form of solution/engine.py:1498-1547). Tokens are taken supervised
        first, in blocks of up to head_chunk rows; within a block the vocabulary is walked in
        chunks small enough that a chunk's logits stay in L2 between the kernels that use them
        (VocabHead): no [rows, V] logits buffer exists. Returns (dh in head order, loss)."""
        n, H = h.shape
        dev, dt = self.device, self.dtype
        order = packed.head_order
        n_sup = packed.n_supervised
        hp = ops.gather_rows(h, order)
        targets = packed.targets.index_select(0, order)
        _, hn, _, _, rstd, _, _ = ops.rms_fwd(hp, self.norm_w, self.eps, dtype=dt)
        tok_loss = torch.empty((n,), device=dev, dtype=torch.float32)
        entropy = torch.empty((n,), device=dev, dtype=torch.float32)
        correct = torch.empty((n,), device=dev, dtype=torch.int32)
        dhp = torch.empty_like(hp)
        if n_sup < n:
            dhp[n_sup:].zero_()
        inv = 1.0 / denom if denom else float("nan")  # 0 / 0, as in the base
        for r0 in range(0, n, self.head_chunk):
            r1 = min(n, r0 + self.head_chunk)
            sup = max(0, min(r1, n_sup) - r0)
            dhn = self.head.block(hn[r0:r1], targets[r0:r1], sup, tok_loss[r0:r1],
                                  entropy[r0:r1], correct[r0:r1])
            if sup:
                ops.rms_bwd(dhn, hp[r0:r0 + sup], rstd[r0:r0 + sup], self.norm_w, dtype=dt,
                            grad_scale=inv, out=dhp[r0:r0 + sup])
        stats.order, stats.tok_loss, stats.entropy, stats.correct = order, tok_loss, entropy, correct
        return dhp, tok_loss.sum() * inv

    def run_layer(self, index, packed, drop, h, dh3):
        """One decoder layer forward and backward through the layer ABI (ql_layer_forward,
        ql_layer_backward), outside a training step: the layer-level parity tests and
        microbenchmarks. packed: the batch's Packed; drop: its ops.Drop for this layer; h, dh3:
        the layer's input and upstream gradient, [n, H] fp32 on the device. Returns (h3, dh,
        [dAq, dBq, dAv, dBv]); the generator and the step's state are not touched."""
        spec, desc = self.layers[index], self.descs[index]
        n, H = h.shape
        with torch.no_grad():
            torch._foreach_copy_(self.lora_views, self.lora_fp32)
        cos, sin = self.rope.table(max(packed.max_len, 1))
        self._set_step(desc, packed, drop, cos, sin)
        arena = _SavedArena(n, spec, 1, self.dtype, self.device)
        arena.h(0).copy_(h)
        sv = arena.saved(0)
        if self.w16 is not None:
            self._dequant_all()
            sv.w16 = self.w16[index * self.weight_elems:].data_ptr()
            sv.w16_ready = 1
        ws = self._workspace_for(desc)
        if self.wstream is not None:
            self.wstream.use(index)
        _lib.call("ql_layer_forward", ctypes.addressof(desc), ctypes.addressof(sv),
                  arena.h(1).data_ptr(), ws.data_ptr(), ws.numel(), ops.stream_ptr())
        h3 = arena.h(1).clone()
        grads = torch.zeros(self.offsets[4 * index + 4] - self.offsets[4 * index],
                            device=self.device, dtype=torch.float32)
        dh3 = dh3.contiguous().float()
        dh3_16 = dh3.to(self.dtype)
        dh = torch.empty_like(dh3)
        dh16 = torch.empty((n, H), device=self.device, dtype=self.dtype)
        _lib.call("ql_layer_backward", ctypes.addressof(desc), ctypes.addressof(sv),
                  dh3.data_ptr(), dh3_16.data_ptr(), grads.data_ptr(),
                  dh.data_ptr(), dh16.data_ptr(), ws.data_ptr(), ws.numel(), ops.stream_ptr())
        if self.wstream is not None:
            self.wstream.done(index)
        views, at = [], 0
        for t in self.lora_fp32[4 * index:4 * index + 4]:
            views.append(grads[at:at + t.numel()].view(t.shape))
            at += t.numel()
        return h3, dh, views

    # -----------------------------------------------------------------------------------------
    # backward
    # -----------------------------------------------------------------------------------------
    def _backward(self, packed, saved, dhp, grad):
        n = packed.n
        H = self.layers[0].H
        arena, (saved_arr, drops), offload = saved
        plan = arena.plan
        if arena.owned:  # the next forward may reuse the arena (queued after this backward)
            self._arena_busy = False
        grads = torch.zeros(self.lora_total, device=self.device, dtype=torch.float32)
        # one view per LoRA weight, made in one call (the buffer is laid out in lora_fp32 order)
        views = list(_unflatten_dense_tensors(grads, self.lora_fp32))
        reducer = None
        if self.data_parallel:
            from .dist import GradReducer

            reducer = GradReducer(self.process_group)
        if n:
            cos, sin = self.rope.table(max(packed.max_len, 1))
            dh = [torch.empty((n, H), device=self.device, dtype=torch.float32) for _ in range(2)]
            dh16 = [torch.empty((n, H), device=self.device, dtype=self.dtype) for _ in range(2)]
            g = grad.detach().float().reshape(1).contiguous()
            ops.scatter_rows(dhp, packed.head_order, dh[0], scale=g, out16=dh16[0])
            cur = 0
            if offload is not None:
                offload.start_backward()
            L = len(self.layers)
            self._set_all_steps(packed, drops, cos, sin)
            wst = self.wstream
            one_call = all(m == memory.KEEP for m in plan.modes) and wst is None
            if one_call:
                # every saved set and weight is in HBM: the whole backward in one call
                ws = self._workspace_for(self.descs[0])
                _lib.call("ql_layers_backward", ctypes.addressof(self.desc_array),
                          ctypes.addressof(saved_arr), L, dh[0].data_ptr(), dh16[0].data_ptr(),
                          dh[1].data_ptr(), dh16[1].data_ptr(), grads.data_ptr(),
                          ctypes.addressof(self._grad_offsets), 1, ws.data_ptr(), ws.numel(),
                          ops.stream_ptr())
            for spec in reversed(self.layers if not one_call else []):
                i = spec.index
                desc = self.descs[i]
                sv, drop = saved_arr[i], drops[i]
                if wst is not None:  # layer i's NF4 bytes in its slot, layer i - 1's on the way
                    wst.use(i, i - 1 if i > 0 else None)
                if plan.modes[i] == memory.RECOMPUTE:
                    self._recompute(i, desc, sv, arena)
                elif plan.modes[i] == memory.OFFLOAD:
                    offload.before_backward(i)
                ws = self._workspace_for(desc)
                lo = self.offsets[4 * i]
                nxt = 1 - cur
                need = i > 0  # the first layer's input is the frozen embedding
                _lib.call("ql_layer_backward", ctypes.addressof(desc), ctypes.addressof(sv),
                          dh[cur].data_ptr(), dh16[cur].data_ptr(), grads[lo:].data_ptr(),
                          dh[nxt].data_ptr() if need else None,
                          dh16[nxt].data_ptr() if need else None, ws.data_ptr(), ws.numel(),
                          ops.stream_ptr())
                if wst is not None:
                    wst.done(i)
                if offload is not None and plan.modes[i] == memory.OFFLOAD:
                    offload.after_backward(i)
                cur = nxt
        if reducer is not None:  # one all-reduce of every LoRA gradient, after the backward
            # through a buffer that keeps its address from step to step (NCCL registers it once);
            # the gradients handed to autograd stay this step's own tensors
            if self._comm is None:
                self._comm = torch.empty_like(grads)
            self._comm.copy_(grads)
            reducer.launch(self._comm)
            reducer.finish(self._comm)
            grads.copy_(self._comm)
        self.last_offload_bytes = offload.bytes_moved if offload is not None else 0
        self.last_offload = offload
        if self._step_events is not None:
            self._step_events[1].record()
        return views


class VocabHead:
    """The lm_head + cross-entropy over the vocabulary in chunks, for a block of head rows (the
    vocabulary-piece form of the reference's head, solution/engine.py:1498-1547 and
    solution/kernels.py:401-479, with pieces sized for L2 instead of streamed from the host):
      (1) logits of the chunk = hn . W_chunk^T on the tensor cores (16-bit, into a chunk buffer
          that stays in L2 until (3) has read it);
      (2) ce_piece: each row's online max / sum exp / sum exp * x / argmax carried across the
          chunks; exp(x - running max) written over the supervised rows' logits; the target's
          weight row copied; the fp32 gradient accumulator moved to the new max with the previous
          chunk's product folded in, acc = alpha (acc + part);
      (3) part = exp(x - max) . W_chunk on the tensor cores (fp32, split-K allowed: the GEMM never
          reads its output).
    ce_finish then gives loss, entropy, accuracy and dhn = (acc + part) / sum - W_target.
    W is read from HBM once per chunk (the second GEMM finds it in L2); no [rows, V] logits
    buffer exists. Buffers grow to the largest block seen and are reused from step to step."""

    def __init__(self, lm_w, dtype, l2_bytes=HEAD_L2_BYTES):
        self.lm_w, self.dtype, self.l2_bytes = lm_w, dtype, l2_bytes
        self.V, self.H = lm_w.shape
        self.device = lm_w.device
        self._buf = None
        # the per-row state's starting value (max, sum, sum x e^x, best): made once here, since
        # a device tensor built from host values waits for the device
        self._init = torch.tensor([float("-inf"), 0.0, 0.0, float("-inf")]).to(self.device)

    def chunk_width(self, rows):
        """Vocabulary entries per chunk: as many as keep the chunk's 16-bit logits within
        l2_bytes, in multiples of 64, evened out over the chunks."""
        def cdiv(a, b):
            return -(-a // b)

        esize = torch.empty((), dtype=self.dtype).element_size()
        width = max(1024, self.l2_bytes // (esize * max(rows, 1)) // 64 * 64)
        return cdiv(cdiv(self.V, cdiv(self.V, width)), 64) * 64

    def _buffers(self, rows, width, sup):
        """The block's buffers, grown (by a quarter more than asked, so that slightly larger
        blocks later reuse them) only when a block needs more rows, logits or supervised rows
        than any before."""
        H, dt, dev = self.H, self.dtype, self.device
        b = self._buf
        need = (rows, rows * width, sup)
        if b is None or any(x < y for x, y in zip(b["shape"], need)):
            rows_, logits_, sup_ = (max(x, y + y // 4) if x < y else x
                                    for x, y in zip(b["shape"] if b else (0, 0, 0), need))
            b = {"shape": (rows_, logits_, sup_),
                 "logits": torch.empty(logits_, device=dev, dtype=dt),
                 "state": torch.empty((rows_, 4), device=dev, dtype=torch.float32),
                 "best": torch.empty(rows_, device=dev, dtype=torch.int64),
                 "xt": torch.empty(rows_, device=dev, dtype=torch.float32),
                 "alpha": torch.empty(max(sup_, 1), device=dev, dtype=torch.float32),
                 "acc": torch.empty((max(sup_, 1), H), device=dev, dtype=torch.float32),
                 "part": torch.empty((max(sup_, 1), H), device=dev, dtype=torch.float32),
                 "wt": torch.empty((max(sup_, 1), H), device=dev, dtype=dt),
                 "dhn": torch.empty((max(sup_, 1), H), device=dev, dtype=dt)}
            self._buf = b
        return b

    def block(self, hn, targets, sup, tok_loss, entropy, correct):
        """One block of head rows hn [rows, H] (16-bit, the first `sup` rows have a target):
        writes tok_loss / entropy / correct [rows] and returns dhn [sup, H] (16-bit), the
        gradient of the summed token losses w.r.t. hn."""
        rows, H = hn.shape
        width = self.chunk_width(rows)
        b = self._buffers(rows, width, sup)
        state, best, xt = b["state"][:rows], b["best"][:rows], b["xt"][:rows]
        state.copy_(self._init.expand(rows, 4))
        logits = b["logits"][:rows * width].view(rows, width)
        acc = b["acc"][:sup] if sup else None
        part = b["part"][:sup] if sup else None
        wt, dhn = b["wt"][:sup], b["dhn"][:sup]
        for v0 in range(0, self.V, width):
            w = min(width, self.V - v0)
            W = self.lm_w[v0:v0 + w]
            chunk = logits[:, :w]
            ops.gemm(hn, W, out=chunk)
            ops.ce_piece(chunk, W, targets, state, best, xt, b["alpha"], wt, v0, sup, acc=acc,
                         part=part, part_valid=v0 > 0 and sup > 0, H=H)
            if sup:
                ops.gemm(chunk[:sup], W, out=part, b_kn=True)
        ops.ce_finish(state, best, xt, targets, tok_loss, entropy, correct, b["acc"], wt, dhn,
                      sup, part=part)
        return dhn


class _SavedArena:
    """One device allocation per step for every layer's saved activations (ql_layer_saved) and
    the residual stream between layers (L + 1 fp32 [n, H] slots)."""

    def __init__(self, n, spec, layers, dtype, device, reuse=None, plan=None):
        self.owned = False
        e = torch.empty((), dtype=dtype).element_size()
        self.layer_bytes, self.fields = memory.saved_set_bytes(n, spec.H, spec.HQ, spec.HKV,
                                                               spec.D, spec.I, e)
        H = spec.H
        self.plan = plan if plan is not None else memory.MemoryPlan([memory.KEEP] * layers)
        self.slots = self.plan.slots  # saved sets in HBM: kept layers + the spill ring
        self.h_bytes = (n * H * 4 + 255) // 256 * 256
        self.layers, self.n, self.H = layers, n, H
        total = max(self.slots * self.layer_bytes + (layers + 1) * self.h_bytes, 256)
        if reuse is not None and reuse.numel() >= total:
            self.buf = reuse
        else:  # grow by a quarter beyond the need, so slightly longer steps still fit
            self.buf = torch.empty(total + total // 4 if reuse is not None else total,
                                   device=device, dtype=torch.uint8)
        self.base = self.buf.data_ptr()

    def h(self, i):
        """Residual stream slot i: the input of layer i (slot L: the head's input)."""
        start = self.slots * self.layer_bytes + i * self.h_bytes
        return self.buf[start:start + self.n * self.H * 4].view(torch.float32).view(self.n, self.H)

    def slot_base(self, i):
        """Device address of layer i's saved set (its own slot, or its ring slot)."""
        return self.base + self.plan.slot(i) * self.layer_bytes

    def saved(self, i):
        b = self.slot_base(i)
        fields = {k: b + off for k, off in self.fields.items()}
        fields["h"] = self.h(i).data_ptr()
        return _lib.struct("ql_layer_saved", **fields)


class _Offload:
    """Offload of spilled layers' saved sets to pinned host memory: the forward's set of layer
    i leaves its ring slot on a copy stream right after the layer (the slot is reused two
    offloaded layers later, after that copy), and the backward brings each set back into a ring
    slot one offloaded layer ahead of its use (the slot is free once the layer that used it is
    done). The last two offloaded layers of the forward stay in their ring slots (no later
    layer reuses them, and the backward needs them first): they make no round trip, so no copy
    sits between the end of the forward and the start of the backward. One cudaMemcpyAsync per
    layer and direction; events order the two streams."""

    def __init__(self, engine, arena, plan):
        self.arena, self.plan = arena, plan
        offloaded = [i for i in plan.spilled() if plan.modes[i] == memory.OFFLOAD]
        self.resident = set(offloaded[-2:])  # ring slots 0 and 1 hold them into the backward
        self.spilled = [i for i in offloaded if i not in self.resident]
        self.order = sorted(offloaded, reverse=True)  # the backward's order
        nbytes = len(self.spilled) * arena.layer_bytes
        if engine._host_ring is None or engine._host_ring.numel() < nbytes:
            # grown with half again as much headroom: pinning gigabytes of host memory takes
            # seconds (and can wait for the GPU), so only a step well above every earlier one
            # may pay it, never each step that is slightly longer than the last
            engine._host_ring = None
            engine._host_ring = torch.empty(nbytes + nbytes // 2, dtype=torch.uint8,
                                            pin_memory=True)
        if engine._copy_stream is None:
            engine._copy_stream = torch.cuda.Stream(device=engine.device)
        self.host, self.stream = engine._host_ring, engine._copy_stream
        self.index = {i: k for k, i in enumerate(self.spilled)}
        self.slot_free = {}   # ring slot -> event after which it may be overwritten
        self.arrived = {}     # layer -> event: its set is back in HBM
        self.bytes_moved = 0
        self.copy_events = []  # (start, end) timing events of every copy, on the copy stream

    def _dev(self, i):
        lb = self.arena.layer_bytes
        off = self.arena.plan.slot(i) * lb
        return self.arena.buf[off:off + lb]

    def _host(self, i):
        lb = self.arena.layer_bytes
        k = self.index[i]
        return self.host[k * lb:(k + 1) * lb]

    def before_forward(self, i):
        if i in self.index or i in self.resident:
            ev = self.slot_free.get(self.plan.slot(i))
            if ev is not None:
                torch.cuda.current_stream().wait_event(ev)

    def after_forward(self, i):
        if i not in self.index:
            return
        done = torch.cuda.Event()
        done.record()
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(done)
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(self.stream)
            self._host(i).copy_(self._dev(i), non_blocking=True)
            out = torch.cuda.Event(enable_timing=True)
            out.record(self.stream)
            self.copy_events.append((t0, out))
        self.slot_free[self.plan.slot(i)] = out
        self.bytes_moved += self.arena.layer_bytes

    def _fetch(self, i):
        ev = self.slot_free.get(self.plan.slot(i))
        with torch.cuda.stream(self.stream):
            if ev is not None:
                self.stream.wait_event(ev)
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(self.stream)
            self._dev(i).copy_(self._host(i), non_blocking=True)
            got = torch.cuda.Event(enable_timing=True)
            got.record(self.stream)
            self.copy_events.append((t0, got))
        self.arrived[i] = got
        self.bytes_moved += self.arena.layer_bytes

    def copy_ms(self):
        """Milliseconds the copy stream spent copying this step (after the copies finished)."""
        return sum(a.elapsed_time(b) for a, b in self.copy_events)

    def start_backward(self):
        # the ring slots' last forward copies must finish before the backward refills them
        for ev in self.slot_free.values():
            self.stream.wait_event(ev)
        self.slot_free = {}
        # the first offloaded layers of the backward are resident; a fetch is only needed first
        # if a single ring slot holds a resident layer (then the next set goes into the other)
        if self.order and self.order[0] not in self.resident:
            self._fetch(self.order[0])

    def before_backward(self, i):
        if i in self.arrived:
            torch.cuda.current_stream().wait_event(self.arrived.pop(i))
        k = self.order.index(i)
        # the next offloaded layer into the slot the previous one used (free once that layer's
        # backward is done): resident layers need no fetch
        if k + 1 < len(self.order) and self.order[k + 1] not in self.resident:
            self._fetch(self.order[k + 1])

    def after_backward(self, i):
        done = torch.cuda.Event()
        done.record()
        self.slot_free[self.plan.slot(i)] = done


class _FusedStep(torch.autograd.Function):
    """The whole model as one autograd node: its inputs are the fp32 LoRA weights, its output the
    loss; backward returns their gradients (the frozen base gets none)."""

    @staticmethod
    def forward(ctx, engine, packed, denom, stats, *lora):
        torch.cuda.nvtx.range_push("qlora_fwd")
        try:
            loss, saved, dhp = engine._forward(packed, denom, stats)
        finally:
            torch.cuda.nvtx.range_pop()
        ctx.engine, ctx.packed, ctx.saved, ctx.dhp = engine, packed, saved, dhp
        return loss

    @staticmethod
    def backward(ctx, grad):
        torch.cuda.nvtx.range_push("qlora_bwd")
        try:
            grads = ctx.engine._backward(ctx.packed, ctx.saved, ctx.dhp, grad)
        finally:
            torch.cuda.nvtx.range_pop()
        ctx.saved = ctx.dhp = None
        return (None, None, None, None, *grads)

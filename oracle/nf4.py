"""NF4 (bitsandbytes layout) quantisation and dequantisation in numpy — test oracle.

Layout (solution/kernels.py:33-41, 79-105): element i of a [rows, cols] weight lives in byte
i // 2, high nibble for even i; one absmax per block of 64 consecutive elements. Dequantised
value = level[nibble] * scale (fp32 product, rounded once to the output type). Nested scale
(double quantisation, solution/kernels.py:85-92): code2[q] * absmax2[b // bs2] rounded to fp32,
then + offset[segment] rounded (two operations, no fused multiply-add).
"""

import numpy as np

# The 16 NF4 levels (QLoRA, Dettmers et al. 2023), as listed at solution/kernels.py:38-41.
NF4_LEVELS = np.array(
    [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
     -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
     0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
     0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], dtype=np.float32)

BS1 = 64


def nested_code():
    """A signed 256-level table for the double-quantised absmax (not bitsandbytes' dynamic map,
    which is absent here: the dequantisation formula does not depend on the table's values)."""
    pos = np.geomspace(1e-4, 1.0, 127, dtype=np.float64)
    code = np.concatenate([-pos[::-1], [0.0], pos, [1.0]]).astype(np.float32)
    return np.sort(code)


class QuantState:
    """The pieces a bitsandbytes Params4bit quant_state holds, as numpy arrays."""

    def __init__(self, packed, absmax, shape, nested=False, code2=None, absmax2=None,
                 offset=None, bs2=256):
        self.packed, self.absmax, self.shape = packed, absmax, tuple(shape)
        self.nested, self.code2, self.absmax2, self.offset, self.bs2 = (
            nested, code2, absmax2, offset, bs2)
        self.code = NF4_LEVELS.copy()


def quantize_nf4(w, nested=False, bs2=256):
    """w: fp32 [rows, cols] -> QuantState. Nearest NF4 level of w / absmax per 64-block."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    flat = w.reshape(-1)
    assert flat.size % BS1 == 0
    blocks = flat.reshape(-1, BS1)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    safe = np.where(absmax > 0, absmax, np.float32(1.0))
    norm = blocks / safe[:, None]
    mids = (NF4_LEVELS[1:] + NF4_LEVELS[:-1]) / 2
    q = np.searchsorted(mids, norm.reshape(-1)).astype(np.uint8)
    packed = ((q[0::2] << 4) | q[1::2]).astype(np.uint8)
    if not nested:
        return QuantState(packed, absmax, (rows, cols))
    offset = np.float32(absmax.mean())
    centred = (absmax - offset).astype(np.float32)
    nb2 = -(-centred.size // bs2)
    padded = np.zeros(nb2 * bs2, np.float32)
    padded[:centred.size] = centred
    absmax2 = np.abs(padded.reshape(nb2, bs2)).max(axis=1).astype(np.float32)
    absmax2 = np.where(absmax2 > 0, absmax2, np.float32(1.0)).astype(np.float32)
    code2 = nested_code()
    normed = centred / np.repeat(absmax2, bs2)[:centred.size]
    mids2 = (code2[1:] + code2[:-1]) / 2
    q2 = np.searchsorted(mids2, normed).astype(np.uint8)
    return QuantState(packed, q2, (rows, cols), nested=True, code2=code2, absmax2=absmax2,
                      offset=np.array([offset], np.float32), bs2=bs2)


def block_scales(st, seg_bounds=None, offsets=None):
    """fp32 scale of every 64-block (nested: code2[q] * absmax2 rounded, + offset rounded)."""
    if not st.nested:
        return st.absmax.astype(np.float32)
    nblk = st.absmax.size
    b = np.arange(nblk)
    prod = (st.code2[st.absmax.astype(np.int64)] * st.absmax2[b // st.bs2]).astype(np.float32)
    if offsets is None:
        off = np.full(nblk, st.offset[0], np.float32)
    else:
        seg = np.zeros(nblk, np.int64)
        for bound in seg_bounds:
            seg += (b >= bound)
        off = np.asarray(offsets, np.float32)[seg]
    return (prod + off).astype(np.float32)


def f32_to_bf16_bits(x):
    """Round-to-nearest-even fp32 -> bf16, as uint16 bits (NaN not handled: none occur here)."""
    u = np.asarray(x, np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))
    return (rounded >> 16).astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequant_nf4(st, out_dtype="f16", seg_bounds=None, offsets=None):
    """QuantState -> [rows, cols] values: np.float16 for "f16", uint16 bf16 bits for "bf16"."""
    scales = block_scales(st, seg_bounds, offsets)
    q = np.empty(st.packed.size * 2, np.uint8)
    q[0::2] = st.packed >> 4
    q[1::2] = st.packed & 15
    vals = (st.code[q].reshape(-1, BS1) * scales[:, None]).astype(np.float32).reshape(st.shape)
    if out_dtype == "f16":
        return vals.astype(np.float16)
    return f32_to_bf16_bits(vals)

"""PyTorch's CUDA dropout keep mask, restated in numpy — test oracle.

Follows solution/kernels.py:108-126 (`_torch_dropout_keep`) and solution/engine.py:767-805
(`TorchDropout.draw`): element e of a contiguous dropout input drawn by thread
t = (e // VEC) % G of G = blocks * 256 threads, at counter ctr + (e // VEC // G) * (VEC / 4)
+ (e % VEC) // 4, component e % 4 of Philox4x32-10(key = seed, counter = (c_lo, c_hi, t, 0));
kept iff u * 2^-32 + 2^-33 < 1 - p in fp32.

Philox4x32-10 is written from the published description (Salmon, Moraes, Dror, Shaw,
"Parallel random numbers: as easy as 1, 2, 3", SC'11): ten rounds of two 32x32->64-bit
multiplies with multipliers 0xD2511F53 / 0xCD9E8D57, key bumped by the Weyl constants
0x9E3779B9 / 0xBB67AE85 between rounds.
"""

import numpy as np

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
MASK32 = np.uint64(0xFFFFFFFF)

BLOCK, UNROLL = 256, 4  # PyTorch Dropout.cu launch constants


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32-10 over uint32 arrays; returns the four output words."""
    c0, c1, c2, c3 = (np.asarray(c, np.uint32).copy() for c in (c0, c1, c2, c3))
    k0 = np.asarray(k0, np.uint32).copy()
    k1 = np.asarray(k1, np.uint32).copy()
    with np.errstate(over="ignore"):
        for r in range(10):
            p0 = M0 * c0.astype(np.uint64)
            p1 = M1 * c2.astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & MASK32).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & MASK32).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
            if r < 9:
                k0 = (k0 + W0).astype(np.uint32)
                k1 = (k1 + W1).astype(np.uint32)
    return c0, c1, c2, c3


def dropout_keep(elems, seed, ctr, threads, p, vec=4):
    """Keep mask (bool) of the given element indices of one dropout call."""
    e = np.asarray(elems, np.int64)
    g = e // vec
    thread = (g % threads).astype(np.uint32)
    c = (np.int64(ctr) + (g // threads) * (vec // 4) + (e % vec) // 4).astype(np.uint64)
    seed_u = np.uint64(seed % (1 << 64))
    k0 = np.full(e.shape, seed_u & MASK32, np.uint64).astype(np.uint32)
    k1 = np.full(e.shape, seed_u >> np.uint64(32), np.uint64).astype(np.uint32)
    r = philox4x32_10((c & MASK32).astype(np.uint32), (c >> np.uint64(32)).astype(np.uint32),
                      thread, np.zeros_like(thread), k0, k1)
    comp = e % 4
    u = np.choose(comp, r)
    uf = u.astype(np.float32) * np.float32(2.3283064365386963e-10) + np.float32(1.1641532182693481e-10)
    return uf.astype(np.float32) < np.float32(1.0 - p)


def draw(nelem, offset, seed, max_blocks, vec=4):
    """TorchDropout.draw (solution/engine.py:787-797): (seed, counter, threads, new offset) of a
    dropout call on nelem elements, for a device with max_blocks resident 256-thread blocks."""
    assert nelem % vec == 0
    blocks = min(max_blocks, (nelem + BLOCK - 1) // BLOCK)
    increment = ((nelem - 1) // (BLOCK * blocks * UNROLL) + 1) * UNROLL
    s = seed - (1 << 64) if seed >= (1 << 63) else seed
    return s, offset // 4, blocks * BLOCK, offset + increment

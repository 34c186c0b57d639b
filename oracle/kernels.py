"""numpy restatements of the reference's elementwise kernels — test oracle (fp32 math, 16-bit
rounding where the reference stores 16-bit values). Each follows the Triton kernel cited; the
golden fixtures in tests/golden (the reference kernels' own outputs) pin them.
"""

import numpy as np

from .philox import dropout_keep

F32 = np.float32


def _f16(x):
    return np.asarray(x, F32).astype(np.float16).astype(F32)


def rms_fwd(x, w, eps, delta=None, tok=None, p=0.0, seed=0, ctr_q=0, ctr_v=0, G=1, vec=4):
    """solution/kernels.py:145-175. Returns xsum, y, yq, yv (fp16 values as fp32), rstd."""
    x = np.asarray(x, F32)
    if delta is not None:
        x = (x + np.asarray(delta, F32)).astype(F32)
    n, H = x.shape
    rstd = (F32(1.0) / np.sqrt((x * x).sum(1, dtype=F32) / F32(H) + F32(eps))).astype(F32)
    y = (np.asarray(w, F32)[None, :] * (x * rstd[:, None])).astype(F32)
    out = {"xsum": x, "y": _f16(y), "rstd": rstd}
    if tok is not None:
        elems = np.asarray(tok, np.int64)[:, None] * H + np.arange(H)[None, :]
        scale = F32(1.0 / (1.0 - p))
        for name, ctr in (("yq", ctr_q), ("yv", ctr_v)):
            keep = dropout_keep(elems.reshape(-1), seed, ctr, G, p, vec).reshape(n, H)
            out[name] = _f16(np.where(keep, y * scale, F32(0)))
    return out


def rms_bwd(dy, x, rstd, w, dres=None, tq=None, tv=None, tok=None, p=0.0, seed=0, ctr_q=0,
            ctr_v=0, G=1, vec=4, grad_scale=1.0):
    """solution/kernels.py:178-205."""
    dy = np.asarray(dy, F32).copy()
    x = np.asarray(x, F32)
    n, H = x.shape
    if tok is not None:
        elems = np.asarray(tok, np.int64)[:, None] * H + np.arange(H)[None, :]
        scale = F32(1.0 / (1.0 - p))
        for t, ctr in ((tq, ctr_q), (tv, ctr_v)):
            if t is None:
                continue
            keep = dropout_keep(elems.reshape(-1), seed, ctr, G, p, vec).reshape(n, H)
            dy = dy + np.where(keep, np.asarray(t, F32) * scale, F32(0))
    g = dy * np.asarray(w, F32)[None, :]
    xhat = x * np.asarray(rstd, F32)[:, None]
    mean = (g * xhat).sum(1, dtype=F32) / F32(H)
    dx = (np.asarray(rstd, F32)[:, None] * (g - xhat * mean[:, None]) * F32(grad_scale)).astype(F32)
    if dres is not None:
        dx = dx + np.asarray(dres, F32)
    return dx


def rope_fwd(qkv, cos, sin, pos, HQ, HKV, D, scale, lq=None, lv=None):
    """solution/kernels.py:212-264, k / v per KV head (not expanded)."""
    qkv = np.asarray(qkv, F32)
    n = qkv.shape[0]
    half = D // 2
    c = np.asarray(cos, F32)[np.asarray(pos)][:, None, :]
    s = np.asarray(sin, F32)[np.asarray(pos)][:, None, :]
    q = qkv[:, :HQ * D].reshape(n, HQ, D).copy()
    if lq is not None:
        q = q + np.asarray(lq, F32).reshape(n, HQ, D) * F32(scale)
    k = qkv[:, HQ * D:(HQ + HKV) * D].reshape(n, HKV, D)
    v = qkv[:, (HQ + HKV) * D:].reshape(n, HKV, D).copy()
    if lv is not None:
        v = v + np.asarray(lv, F32).reshape(n, HKV, D) * F32(scale)

    def rot(x):
        x1, x2 = x[..., :half], x[..., half:]
        return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], -1)

    return _f16(rot(q)), _f16(rot(k)), _f16(v)


def rope_bwd(dq, dk, dv, cos, sin, pos, HQ, HKV, D):
    """solution/kernels.py:267-306: dk / dv may be per query head (summed over each group)."""
    dq = np.asarray(dq, F32)
    n = dq.shape[0]
    half = D // 2
    c = np.asarray(cos, F32)[np.asarray(pos)][:, None, :]
    s = np.asarray(sin, F32)[np.asarray(pos)][:, None, :]

    def group_sum(t):
        t = np.asarray(t, F32)
        heads = t.shape[1]
        return t.reshape(n, HKV, heads // HKV, D).sum(2, dtype=F32)

    def rot_t(g):
        g1, g2 = g[..., :half], g[..., half:]
        return np.concatenate([g1 * c + g2 * s, g2 * c - g1 * s], -1)

    out = np.concatenate([rot_t(dq).reshape(n, -1), rot_t(group_sum(dk)).reshape(n, -1),
                          group_sum(dv).reshape(n, -1)], 1)
    return _f16(out)


def glu_fwd(gu):
    """solution/kernels.py:312-321."""
    gu = np.asarray(gu, F32)
    I = gu.shape[1] // 2
    g, u = gu[:, :I], gu[:, I:]
    return _f16(g / (F32(1) + np.exp(-g)) * u)


def glu_bwd(dm, gu):
    """solution/kernels.py:324-336: [dL/dg | dL/du]."""
    gu = np.asarray(gu, F32)
    I = gu.shape[1] // 2
    g, u, d = gu[:, :I], gu[:, I:], np.asarray(dm, F32)
    sig = F32(1) / (F32(1) + np.exp(-g))
    return np.concatenate([_f16(d * u * sig * (F32(1) + g * (F32(1) - sig))), _f16(d * g * sig)], 1)


def ce_rows(logits, target):
    """solution/kernels.py:344-388 in float64 accumulation: (loss, entropy, correct, grad)."""
    x = np.asarray(logits, np.float64)
    t = np.asarray(target)
    m = x.max(1, keepdims=True)
    e = np.exp(x - m)
    ssum = e.sum(1, keepdims=True)
    lse = (m + np.log(ssum))[:, 0]
    p = e / ssum
    entropy = lse - (p * x).sum(1)
    valid = t >= 0
    tt = np.where(valid, t, 0)
    xt = x[np.arange(len(t)), tt]
    loss = np.where(valid, lse - xt, 0.0)
    correct = (valid & (x.argmax(1) == t)).astype(np.int32)  # argmax: first maximum
    grad = p.copy()
    grad[np.arange(len(t))[valid], t[valid]] -= 1.0
    grad[~valid] = 0.0
    return loss.astype(F32), entropy.astype(F32), correct, _f16(grad)

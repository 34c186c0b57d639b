"""CPU restatement of the reference's fused training step — test oracle and timed CPU baseline.

Forward follows solution/engine.py:1054-1181 (`_layer_forward`) and 1352-1400 (`_Head`) with the
reference's rounding points: the 16-bit compute type at every projection output, the attention
inputs and output, the MLP product; fp32 for the residual stream, the norms, RoPE, softmax and
the loss. LoRA per solution/engine.py:1088-1093 (xq = drop(a) A^T, lq = xq B^T, both rounded),
dropout masks per solution/kernels.py:108-126 (numpy Philox, oracle/philox.py) drawn in the
reference's order (layer 0 q, layer 0 v, layer 1 q, ...). Attention is per-sequence causal SDPA
math in fp32 (as solution/test_kernels.py:245-281 checks the reference's).

Backward is torch-CPU autograd of that fp32 graph with straight-through roundings: the exact
gradient of the rounded forward, the yardstick the reference's own whole-step test uses against
HF + PEFT (loss rel < 2e-3, LoRA gradients rel-L2 < 2e-2, solution/test_kernels.py:314-359).

Weights come from the model object's NF4 bytes through oracle/nf4.py (numpy), never from the
product's kernels.
"""

import numpy as np
import torch

from .nf4 import QuantState, dequant_nf4, bf16_bits_to_f32
from .philox import dropout_keep, draw


def _np(t):
    return t.detach().cpu().numpy()


def _rounder(dtype):
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16

    def r(x):  # round to the 16-bit type, straight-through gradient
        return x + (x.to(tdt).float() - x).detach()

    return r


def _dequant_param(param, dtype):
    qs = param.quant_state
    st = QuantState(_np(param.data).reshape(-1).astype(np.uint8), _np(qs.absmax), tuple(qs.shape),
                    nested=bool(qs.nested),
                    code2=_np(qs.state2.code).astype(np.float32) if qs.nested else None,
                    absmax2=_np(qs.state2.absmax).astype(np.float32) if qs.nested else None,
                    offset=np.array([float(qs.offset)], np.float32) if qs.nested else None,
                    bs2=int(qs.state2.blocksize) if qs.nested else 256)
    st.code = _np(qs.code).astype(np.float32)
    out = dequant_nf4(st, dtype)
    vals = out.astype(np.float32) if dtype == "f16" else bf16_bits_to_f32(out)
    return torch.from_numpy(vals)


def weights_from_model(model, dtype="f16"):
    """fp32 CPU copies of everything the step reads, NF4 weights dequantised by the oracle."""
    return weights_from_model_layers(model, None, dtype)


def weights_from_model_layers(model, which, dtype="f16", embed=None, norm=None):
    """weights_from_model restricted to the decoder layers listed in `which` (None: all).
    embed / norm: fp32 CPU copies of the (tied) embedding and the final norm weight already at
    hand, used instead of copying them again."""
    causal = model.get_base_model()
    inner = causal.model
    cfg = causal.config
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    layers = []
    for li, layer in enumerate(inner.layers):
        if which is not None and li not in which:
            continue
        attn, mlp = layer.self_attn, layer.mlp
        base = lambda m: getattr(m, "base_layer", m)  # noqa: E731
        d = {}
        for name, mod in (("q", attn.q_proj), ("k", attn.k_proj), ("v", attn.v_proj),
                          ("o", attn.o_proj), ("gate", mlp.gate_proj), ("up", mlp.up_proj),
                          ("down", mlp.down_proj)):
            d["W" + name] = _dequant_param(base(mod).weight, dtype)
        d["bias"] = torch.cat([base(m).bias.detach().to(tdt).float().cpu()
                               for m in (attn.q_proj, attn.k_proj, attn.v_proj)])
        d["ln1"] = layer.input_layernorm.weight.detach().float().cpu()
        d["ln2"] = layer.post_attention_layernorm.weight.detach().float().cpu()
        for short, mod in (("q", attn.q_proj), ("v", attn.v_proj)):
            name = mod.active_adapters[0]
            d["A" + short] = mod.lora_A[name].weight.detach().float().cpu()
            d["B" + short] = mod.lora_B[name].weight.detach().float().cpu()
            d["s"] = float(mod.scaling[name])
            d["p"] = float(mod.lora_dropout[name].p)
        d["eps"] = float(layer.input_layernorm.variance_epsilon)
        layers.append(d)
    if embed is None:
        embed = inner.embed_tokens.weight.detach().to(tdt).float().cpu()
        lm = causal.lm_head.weight.detach().to(tdt).float().cpu()
    else:
        lm = embed
    return {
        "layers": layers,
        "embed": embed,
        "lm": lm,
        "norm": norm if norm is not None else inner.norm.weight.detach().float().cpu(),
        "eps": float(inner.norm.variance_epsilon),
        "H": cfg.hidden_size, "HQ": cfg.num_attention_heads, "HKV": cfg.num_key_value_heads,
        "D": cfg.head_dim, "I": cfg.intermediate_size, "theta": cfg.rope_theta,
        "dtype": dtype,
    }


def rope_tables(positions, D, theta):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
    f = positions.float()[:, None] * inv[None, :]
    return f.cos(), f.sin()


def rope(x, cos, sin):
    """Rotate-half RoPE on [n, heads, D] (solution/kernels.py:212-264)."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def causal_attention(q, k, v, lengths, scale):
    """q [n, HQ, D], k / v [n, HKV, D] (fp32 values) -> out [n, HQ, D]; per-sequence causal."""
    HQ, HKV = q.shape[1], k.shape[1]
    group = HQ // HKV
    outs, start = [], 0
    for ln in lengths:
        sl = slice(start, start + ln)
        qs = q[sl].transpose(0, 1)
        ks = k[sl].transpose(0, 1).repeat_interleave(group, 0)
        vs = v[sl].transpose(0, 1).repeat_interleave(group, 0)
        sc = (qs @ ks.transpose(-1, -2)) * scale
        mask = torch.ones(ln, ln, dtype=torch.bool).triu(1)
        sc = sc.masked_fill(mask, float("-inf"))
        outs.append((torch.softmax(sc, -1) @ vs).transpose(0, 1))
        start += ln
    return torch.cat(outs, 0)


class DropState:
    """The CUDA generator state the step starts from, and the device's dropout grid limit."""

    def __init__(self, seed, offset, max_blocks, vec=4):
        self.seed, self.offset, self.max_blocks, self.vec = seed, offset, max_blocks, vec


def decoder_layer(W, L, h, lora, masks, lengths, cos, sin):
    """One decoder layer forward (solution/engine.py:1054-1181): residual h [n, H] fp32 -> h3,
    with the LoRA weights `lora` = [Aq, Bq, Av, Bv] (fp32 tensors, may require grad) and the
    q / v dropout keep masks [n, H] (bool). The 16-bit roundings sit where the reference's
    kernels and fp16 GEMMs put them; differentiable end to end."""
    r = _rounder(W["dtype"])
    H, HQ, HKV, D = W["H"], W["HQ"], W["HKV"], W["D"]
    n = h.shape[0]
    Aq, Bq, Av, Bv = lora
    p, s = L["p"], L["s"]
    keep = 1.0 / (1.0 - p) if p > 0 else 1.0
    rstd = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + L["eps"])
    y = L["ln1"] * (h * rstd)
    a = r(y)
    aq = r(torch.where(masks[0], y * keep, torch.zeros_like(y)))
    av = r(torch.where(masks[1], y * keep, torch.zeros_like(y)))
    Wqkv = torch.cat([L["Wq"], L["Wk"], L["Wv"]])
    qkv = r(a @ Wqkv.t() + L["bias"])
    lq = r(r(aq @ r(Aq).t()) @ r(Bq).t())
    lv = r(r(av @ r(Av).t()) @ r(Bv).t())
    q = qkv[:, :HQ * D] + s * lq
    k = qkv[:, HQ * D:(HQ + HKV) * D]
    v = qkv[:, (HQ + HKV) * D:] + s * lv
    q = r(rope(q.view(n, HQ, D), cos, sin))
    k = r(rope(k.view(n, HKV, D), cos, sin))
    v = r(v.view(n, HKV, D))
    out = r(causal_attention(q, k, v, lengths, D ** -0.5))
    o = r(out.reshape(n, HQ * D) @ L["Wo"].t())
    h2 = h + o
    rstd2 = torch.rsqrt(h2.pow(2).mean(-1, keepdim=True) + L["eps"])
    b = r(L["ln2"] * (h2 * rstd2))
    g = r(b @ L["Wgate"].t())
    u = r(b @ L["Wup"].t())
    m = r(torch.nn.functional.silu(g) * u)
    d = r(m @ L["Wdown"].t())
    return h2 + d


def layer_with_dropout(W, L, h, dh3, lengths, T, drop):
    """One decoder layer forward and backward on a right-padded batch of `lengths` (padded width
    T) with LoRA dropout: drop = (seed, counter of the q call, counter of the v call, threads,
    vec). Returns (h3, dh, [dAq, dBq, dAv, dBv]) — what the reference's _Layer computes
    (solution/engine.py:1184-1340) for upstream gradient dh3."""
    H = W["H"]
    n = h.shape[0]
    pos = torch.cat([torch.arange(x) for x in lengths])
    rows = torch.repeat_interleave(torch.arange(len(lengths)), torch.tensor(lengths))
    tok = rows * T + pos
    cos, sin = rope_tables(pos, W["D"], W["theta"])
    elems = (tok[:, None] * H + torch.arange(H)[None, :]).numpy()
    seed, ctr_q, ctr_v, threads, vec = drop
    masks = [torch.from_numpy(dropout_keep(elems, seed, c, threads, L["p"], vec)).view(n, H)
             for c in (ctr_q, ctr_v)]
    h = h.clone().requires_grad_()
    lora = [L[k].clone().requires_grad_() for k in ("Aq", "Bq", "Av", "Bv")]
    h3 = decoder_layer(W, L, h, lora, masks, lengths, cos, sin)
    grads = torch.autograd.grad(h3, [h] + lora, dh3)
    return h3.detach(), grads[0], list(grads[1:])


def step(W, input_ids, attention_mask, labels, denom, drop_state=None, lora_params=None):
    """One forward + backward. Returns dict(loss, tok_loss, entropy, correct, grads=[dAq, dBq,
    dAv, dBv per layer], offset=the generator offset after the step). Rows in packed order."""
    r = _rounder(W["dtype"])
    ids = torch.as_tensor(np.asarray(input_ids))
    mask = torch.as_tensor(np.asarray(attention_mask)).bool()
    lab = torch.as_tensor(np.asarray(labels))
    B, T = ids.shape
    lengths = mask.sum(1).tolist()
    flat = mask.reshape(-1).nonzero().squeeze(1)
    n = flat.numel()
    pos = flat % T
    shifted = torch.full_like(lab, -100)
    shifted[:, :-1] = lab[:, 1:]
    targets = shifted.reshape(-1)[flat]
    H, HQ, HKV, D = W["H"], W["HQ"], W["HKV"], W["D"]
    cos, sin = rope_tables(pos, D, W["theta"])
    elems = (flat[:, None] * H + torch.arange(H)[None, :]).numpy()
    params = []
    h = W["embed"][ids.reshape(-1)[flat]]
    offset = drop_state.offset if drop_state is not None else 0
    for L in W["layers"]:
        lora = [L[k].clone().requires_grad_() for k in ("Aq", "Bq", "Av", "Bv")]
        params += lora
        masks = []
        for _ in range(2):
            if drop_state is not None and L["p"] > 0:
                seed, ctr, thr, offset = draw(B * T * H, offset, drop_state.seed,
                                              drop_state.max_blocks, drop_state.vec)
                masks.append(torch.from_numpy(dropout_keep(elems, seed, ctr, thr, L["p"],
                                                           drop_state.vec)))
            else:
                masks.append(torch.ones(n, H, dtype=torch.bool))
        h = decoder_layer(W, L, h, lora, masks, lengths, cos, sin)
    rstd = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + W["eps"])
    hn = r(W["norm"] * (h * rstd))
    logits = r(hn @ W["lm"].t())
    lse = torch.logsumexp(logits, -1)
    prob = torch.softmax(logits, -1)
    entropy = (lse - (prob * logits).sum(-1)).detach()
    valid = targets >= 0
    tgt = torch.where(valid, targets, torch.zeros_like(targets))
    xt = logits.gather(1, tgt[:, None])[:, 0]
    tok_loss = torch.where(valid, lse - xt, torch.zeros_like(lse))
    loss = tok_loss.sum() / denom
    grads = torch.autograd.grad(loss, params)
    correct = (valid & (logits.argmax(-1) == targets)).int()
    return {"loss": loss.detach(), "tok_loss": tok_loss.detach(), "entropy": entropy,
            "correct": correct, "grads": [g_.detach() for g_ in grads], "offset": offset,
            "targets": targets, "n": n}


def layer_forward_backward(W, L, h, lengths, pos, dh3):
    """Config 1 of the benchmark (one decoder layer, fp32, no dropout): forward from residual h
    [n, H] and backward of the upstream gradient dh3; returns (h3, dh, LoRA grads). The timed
    CPU baseline of the reference's PyTorch path."""
    r = _rounder(W["dtype"])
    H, HQ, HKV, D = W["H"], W["HQ"], W["HKV"], W["D"]
    n = h.shape[0]
    cos, sin = rope_tables(pos, D, W["theta"])
    h = h.clone().requires_grad_()
    Aq = L["Aq"].clone().requires_grad_()
    Bq = L["Bq"].clone().requires_grad_()
    Av = L["Av"].clone().requires_grad_()
    Bv = L["Bv"].clone().requires_grad_()
    s = L["s"]
    rstd = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + L["eps"])
    a = r(L["ln1"] * (h * rstd))
    Wqkv = torch.cat([L["Wq"], L["Wk"], L["Wv"]])
    qkv = r(a @ Wqkv.t() + L["bias"])
    lq = r(r(a @ r(Aq).t()) @ r(Bq).t())
    lv = r(r(a @ r(Av).t()) @ r(Bv).t())
    q = r(rope((qkv[:, :HQ * D] + s * lq).view(n, HQ, D), cos, sin))
    k = r(rope(qkv[:, HQ * D:(HQ + HKV) * D].reshape(n, HKV, D), cos, sin))
    v = r((qkv[:, (HQ + HKV) * D:] + s * lv).view(n, HKV, D))
    out = r(causal_attention(q, k, v, lengths, D ** -0.5))
    h2 = h + r(out.reshape(n, HQ * D) @ L["Wo"].t())
    rstd2 = torch.rsqrt(h2.pow(2).mean(-1, keepdim=True) + L["eps"])
    b = r(L["ln2"] * (h2 * rstd2))
    m = r(torch.nn.functional.silu(r(b @ L["Wgate"].t())) * r(b @ L["Wup"].t()))
    h3 = h2 + r(m @ L["Wdown"].t())
    grads = torch.autograd.grad(h3, [h, Aq, Bq, Av, Bv], dh3)
    return h3.detach(), grads[0], list(grads[1:])


def head_forward_backward(W, h, ids):
    """The reference head (solution/engine.py:1352-1400) over rows h [n, H] with next-token
    targets ids: final norm, 16-bit logits, cross-entropy, and the gradient w.r.t. h."""
    r = _rounder(W["dtype"])
    h = h.clone().requires_grad_()
    rstd = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + W["eps"])
    hn = r(W["norm"] * (h * rstd))
    logits = r(hn @ W["lm"].t())
    loss = torch.nn.functional.cross_entropy(logits, ids, reduction="sum")
    (dh,) = torch.autograd.grad(loss, h)
    return loss.detach(), dh

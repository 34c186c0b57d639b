"""Generates tests/golden/layer_cfg0.npz: one Qwen2 decoder layer at BASELINE configs[0]'s shapes,
forward and backward, computed by the reference's OWN layer code - `_Layer.apply` of
solution/engine.py:1184-1340 with its `_layer_forward`, `dequant`, `_rms_fwd/_rms_bwd`,
`_rope_fwd/_rope_bwd`, `_glu_fwd/_glu_bwd` and the fp16 torch GEMMs, the Triton kernels of
solution/kernels.py running on CPU tensors under TRITON_INTERPRET=1.

    python tests/golden/make_layer_golden.py /path/to/the/reference/checkout

Run it where the reference is checked out (the build container); the GPU box never reads the
reference, only the fixture. Two calls of the reference cannot run on a CPU and are replaced:
  * `_attn_fwd` / `_attn_bwd` (PyTorch's CUDA memory-efficient varlen attention): per-sequence
    causal attention through torch's scaled_dot_product_attention in fp32, outputs rounded to
    fp16 - the yardstick solution/test_kernels.py:245-281 holds the reference's attention to;
  * `TorchDropout` (reads the CUDA generator and the device's SM count): a stand-in with the
    same draw arithmetic (oracle/philox.draw) from a fixed seed and offset, for a B200's
    148 SMs x 8 resident 256-thread blocks.
Layer: H 1536, 12 / 2 heads, D 128, I 8960, eps 1e-6, theta 1e6, base weights N(0, 0.02) quantised
to NF4 (blocksize 64, fp32 absmax, not double-quantised: the interpreter lacks libdevice.mul_rn,
which the nested path calls), q/k/v bias N(0, 0.02), LoRA r 16 / alpha 32 / dropout 0.05 on q and
v (A Kaiming-uniform, B N(0, 0.02)); 4 sequences with lengths uniform in [64, 256], packed;
input and upstream gradient N(0, 1). Weights come from this repository's model stand-in built on
the CPU with fixed seeds (tests/golden/layer_case.py); the fixture keeps a checksum of the NF4 bytes and of
the inputs so a test can confirm it rebuilt the same ones. Stored: the layer's output minus its
input and the input gradient minus the upstream gradient (fp16: the layer's own contribution,
not swamped by the residual) on every ROW_STRIDE-th token, and the four LoRA weight gradients
(fp32, whole).
"""

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle.philox import draw  # noqa: E402
from tests.golden.layer_case import (DROP_OFFSET, DROP_SEED, FIXTURE, MAX_BLOCKS, P_DROP,  # noqa: E402
                                     VEC, drop_state, layer_config, layer_inputs, layer_model,
                                     nf4_checksum)


def _reference_layer(ref_root):
    sys.path.insert(0, ref_root)
    from solution import engine as E  # the reference's own step (no apply(), no CUDA needed)

    def attn_fwd(q, k, v, packed, scale):
        outs, lses = [], []
        for a, b in zip(packed.cu_seqlens[:-1].tolist(), packed.cu_seqlens[1:].tolist()):
            qs, ks, vs = (t[a:b].float().transpose(0, 1) for t in (q, k, v))
            sc = (qs @ ks.transpose(-1, -2)) * scale
            sc = sc.masked_fill(torch.ones(b - a, b - a, dtype=torch.bool).triu(1), float("-inf"))
            lses.append(torch.logsumexp(sc, -1))
            outs.append(torch.nn.functional.scaled_dot_product_attention(
                qs, ks, vs, is_causal=True, scale=scale).transpose(0, 1))
        return torch.cat(outs).to(torch.float16), lses, None, None

    def attn_bwd(dout, q, k, v, out, lse, seed, offset, packed, scale):
        dq, dk, dv = (torch.empty_like(t) for t in (q, k, v))
        for a, b in zip(packed.cu_seqlens[:-1].tolist(), packed.cu_seqlens[1:].tolist()):
            with torch.enable_grad():  # (autograd runs a Function's backward without grad mode)
                qs, ks, vs = (t[a:b].float().transpose(0, 1).requires_grad_() for t in (q, k, v))
                o = torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=True,
                                                                     scale=scale)
                g = torch.autograd.grad(o, (qs, ks, vs), dout[a:b].float().transpose(0, 1))
            for dst, src in zip((dq, dk, dv), g):
                dst[a:b] = src.transpose(0, 1).to(dst.dtype)
        return dq, dk, dv

    E._attn_fwd, E._attn_bwd = attn_fwd, attn_bwd
    return E


ROW_STRIDE = 2  # tokens of the stored per-token outputs: every second one (a smaller fixture)


class _FixedDropout:
    """TorchDropout's draw arithmetic over a fixed (seed, offset) instead of the CUDA generator."""

    vec = VEC

    def __init__(self):
        self.offset = DROP_OFFSET

    def draw(self, nelem):
        seed, ctr, threads, self.offset = draw(nelem, self.offset, DROP_SEED, MAX_BLOCKS, VEC)
        return seed, ctr, threads


def main():
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    E = _reference_layer(sys.argv[1])
    torch.set_num_threads(os.cpu_count() or 4)
    model = layer_model()
    causal = model.get_base_model()
    layer = causal.model.layers[0]
    cfg = layer_config()
    spec = E.LayerSpec(layer, cfg, {"q": "default", "v": "default"}, 0)
    lengths, T, h, dh3 = layer_inputs()
    B, H = len(lengths), cfg.hidden_size
    mask = (torch.arange(T)[None, :] < torch.tensor(lengths)[:, None]).long()
    ids = torch.zeros(B, T, dtype=torch.int64)
    labels = torch.full((B, T), -100, dtype=torch.int64)
    dropout = _FixedDropout()
    packed = E.Packed(ids, mask, labels, E.RopeTable(causal.model.rotary_emb, cfg.head_dim, "cpu"),
                      dropout, P_DROP)
    q, v = layer.self_attn.q_proj, layer.self_attn.v_proj
    lora = [q.lora_A["default"].weight, q.lora_B["default"].weight,
            v.lora_A["default"].weight, v.lora_B["default"].weight]
    lora = [t.detach().clone().requires_grad_() for t in lora]
    hin = h.clone().requires_grad_()
    h3 = E._Layer.apply(hin, spec, packed, lora[0], lora[1], None, None, lora[2], lora[3])
    torch.autograd.backward(h3, dh3)
    seed, ctr_q, ctr_v, threads, end = drop_state(lengths, T, H)
    assert dropout.offset == end
    out = dict(lengths=np.array(lengths), T=T, drop=np.array([seed, ctr_q, ctr_v, threads, VEC]),
               p=P_DROP, nf4_checksum=nf4_checksum(model), h_sum=float(h.double().sum()),
               dh3_sum=float(dh3.double().sum()),
               row_stride=ROW_STRIDE,
               delta_h=(h3.detach() - h)[::ROW_STRIDE].to(torch.float16).numpy(),
               delta_dh=(hin.grad - dh3)[::ROW_STRIDE].to(torch.float16).numpy(),
               dAq=lora[0].grad.numpy(), dBq=lora[1].grad.numpy(),
               dAv=lora[2].grad.numpy(), dBv=lora[3].grad.numpy())
    np.savez_compressed(FIXTURE, **out)
    print("wrote", FIXTURE, os.path.getsize(FIXTURE), "bytes; n =", sum(lengths))


if __name__ == "__main__":
    main()

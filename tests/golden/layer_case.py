"""The case of tests/golden/layer_cfg0.npz (made by make_layer_golden.py from the reference's own
layer): one Qwen2 decoder layer at BASELINE configs[0]'s shapes. Shared by the generator and the
tests that hold the oracle (CPU) and the CUDA layer (GPU) to the fixture.

Layer: H 1536, 12 / 2 heads, D 128, I 8960, eps 1e-6, theta 1e6, base weights N(0, 0.02) in NF4
(blocksize 64, fp32 absmax), q/k/v bias N(0, 0.02), norm weights 1 + N(0, 0.1), LoRA r 16 /
alpha 32 / dropout 0.05 on q and v (A Kaiming-uniform, B N(0, 0.02)); 4 sequences with lengths
uniform in [64, 256], packed; input and upstream gradient N(0, 1); dropout draws from a fixed
(seed, offset) on a device with 148 SMs x 8 resident 256-thread blocks (a B200).
"""

import os

import numpy as np
import torch

from hack_fe30cb28_opus_5_5_ultracode_b200.model import Qwen2Config, build_qwen2_qlora
from oracle.philox import draw

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "layer_cfg0.npz")
MODEL_SEED, INPUT_SEED, LENGTH_SEED = 11, 12, 13
DROP_SEED, DROP_OFFSET, MAX_BLOCKS, VEC = 424242, 8, 148 * 8, 4
P_DROP = 0.05


def layer_config():
    return Qwen2Config(vocab_size=64, num_hidden_layers=1)


def layer_model():
    """The layer's weights: a one-layer 1.5B-width stand-in model, built on the CPU (so every
    machine draws the same numbers; model.move_to puts it on a GPU)."""
    return build_qwen2_qlora(layer_config(), dropout=P_DROP, device="cpu", seed=MODEL_SEED,
                             nested=False, norm_noise=0.1)


def layer_inputs():
    """(lengths, T, h [n, H] fp32, dh3 [n, H] fp32) on the CPU."""
    rng = np.random.default_rng(LENGTH_SEED)
    lengths = [int(x) for x in rng.integers(64, 257, 4)]
    n, H = sum(lengths), layer_config().hidden_size
    g = torch.Generator().manual_seed(INPUT_SEED)
    h = torch.randn(n, H, generator=g)
    dh3 = torch.randn(n, H, generator=g)
    return lengths, max(lengths), h, dh3


def nf4_checksum(model):
    """Sum of every NF4 byte and absmax of the layer, in float64 (a rebuild check)."""
    layer = model.get_base_model().model.layers[0]
    total = 0.0
    for mod in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj,
                layer.self_attn.o_proj, layer.mlp.gate_proj, layer.mlp.up_proj,
                layer.mlp.down_proj):
        w = getattr(mod, "base_layer", mod).weight
        total += float(w.data.double().sum()) + float(w.quant_state.absmax.double().sum())
    return total


def drop_state(lengths, T, H):
    """(seed, counter of the q call, counter of the v call, threads, generator offset after both)
    of the layer's two dropout draws."""
    nelem = len(lengths) * T * H
    seed, ctr_q, threads, off = draw(nelem, DROP_OFFSET, DROP_SEED, MAX_BLOCKS, VEC)
    _, ctr_v, _, end = draw(nelem, off, DROP_SEED, MAX_BLOCKS, VEC)
    return seed, ctr_q, ctr_v, threads, end

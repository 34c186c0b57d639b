"""One decoder layer at configs[0]'s shapes, forward and backward, against the fixture the
reference's OWN layer produced (tests/golden/make_layer_golden.py: `_Layer.apply` of
solution/engine.py:1184-1340 with its Triton kernels on CPU): the CPU oracle on the CPU, this
library's CUDA layer through the layer ABI on the GPU. Tolerances: the layer's contribution to the
residual and to the input gradient within rel-L2 1e-2, the LoRA weight gradients within rel-L2
1e-2 (north-star bound for LoRA gradients); both sides round to fp16 at the same points, so the
gap is GEMM accumulation order and attention arithmetic."""

import numpy as np
import pytest
import torch

from tests.golden import layer_case as case

TOL = 1e-2


def _rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp(min=1e-30))


@pytest.fixture(scope="module")
def golden():
    g = np.load(case.FIXTURE)
    lengths, T, h, dh3 = case.layer_inputs()
    assert g["lengths"].tolist() == lengths and int(g["T"]) == T
    assert float(g["h_sum"]) == float(h.double().sum())  # the same inputs were rebuilt
    assert float(g["dh3_sum"]) == float(dh3.double().sum())
    return g, lengths, T, h, dh3


def _check(golden_arrays, h, dh3, h3, dh, grads):
    g = golden_arrays
    k = int(g["row_stride"])  # the fixture keeps every k-th token's outputs
    assert _rel((h3 - h)[::k], g["delta_h"].astype(np.float32)) < TOL
    assert _rel((dh - dh3)[::k], g["delta_dh"].astype(np.float32)) < TOL
    for name, got in zip(("dAq", "dBq", "dAv", "dBv"), grads):
        assert _rel(got, g[name]) < TOL, name


def test_oracle_layer_matches_the_reference_layer(golden):
    from oracle import step as oracle_step

    g, lengths, T, h, dh3 = golden
    model = case.layer_model()
    assert case.nf4_checksum(model) == float(g["nf4_checksum"])
    W = oracle_step.weights_from_model(model, "f16")
    seed, ctr_q, ctr_v, threads, vec = (int(x) for x in g["drop"])
    h3, dh, grads = oracle_step.layer_with_dropout(W, W["layers"][0], h, dh3, lengths, T,
                                                   (seed, ctr_q, ctr_v, threads, vec))
    _check(g, h, dh3, h3, dh, grads)


@pytest.mark.gpu
def test_cuda_layer_matches_the_reference_layer(golden):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops
    from hack_fe30cb28_opus_5_5_ultracode_b200.engine import FusedQwen2, Packed
    from hack_fe30cb28_opus_5_5_ultracode_b200.model import move_to

    g, lengths, T, h, dh3 = golden
    dev = torch.device("cuda")
    model = case.layer_model()
    assert case.nf4_checksum(model) == float(g["nf4_checksum"])
    move_to(model, dev)
    engine = FusedQwen2(model, dtype=torch.float16)
    B = len(lengths)
    mask = (torch.arange(T)[None, :] < torch.tensor(lengths)[:, None]).long()
    zeros = torch.zeros(B, T, dtype=torch.int64)
    packed = Packed(zeros.to(dev), mask.to(dev), torch.full_like(zeros, -100).to(dev))
    seed, ctr_q, ctr_v, threads, vec = (int(x) for x in g["drop"])
    drop = ops.Drop(packed.tok, seed, ctr_q, ctr_v, threads, float(g["p"]), vec)
    h3, dh, grads = engine.run_layer(0, packed, drop, h.to(dev), dh3.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    _check(g, h, dh3, h3.cpu(), dh.cpu(), [t.cpu() for t in grads])

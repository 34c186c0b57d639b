"""NF4 dequantisation (bit-exact vs the reference kernel's golden output and the oracle) and the
tcgen05 GEMM (vs a torch fp32 matmul), through the C ABI on the GPU."""

import numpy as np
import pytest
import torch

from oracle.nf4 import bf16_bits_to_f32, dequant_nf4, quantize_nf4

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _W:
    """What ops.nf4_dequant reads from a weight."""

    def __init__(self, st, seg1=2147483647, seg2=2147483647, offsets=None):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
        self.shape = st.shape
        self.packed = t(st.packed)
        self.absmax = t(st.absmax)
        self.code = t(st.code)
        self.nested = st.nested
        self.bs2 = st.bs2 if st.nested else 1
        self.seg1, self.seg2 = seg1, seg2
        if st.nested:
            self.code2 = t(st.code2)
            self.absmax2 = t(st.absmax2)
            self.offsets = t(offsets if offsets is not None else st.offset)
        else:
            self.code2 = self.absmax2 = self.offsets = None


def test_nf4_dequant_matches_reference_golden(golden):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    g = golden("nf4.npz")
    rows, cols = int(g["rows"]), int(g["cols"])

    class St:
        pass

    st = St()
    st.shape, st.packed, st.absmax, st.nested = (rows, cols), g["packed"], g["absmax"], False
    st.bs2 = 1
    from oracle.nf4 import NF4_LEVELS

    st.code = NF4_LEVELS
    out = ops.nf4_dequant(_W(st))
    assert torch.equal(out.cpu(), torch.from_numpy(g["out"]))


@pytest.mark.parametrize("nested", [False, True])
@pytest.mark.parametrize("shape", [(256, 1536), (1536, 512), (17920, 1536), (128, 64)])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_nf4_dequant_matches_oracle(nested, shape, dtype):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    rng = np.random.default_rng(shape[0] + 7 * nested)
    w = (rng.standard_normal(shape) * 0.05).astype(np.float32)
    st = quantize_nf4(w, nested=nested)
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    out = ops.nf4_dequant(_W(st), dtype=tdt)
    ref = dequant_nf4(st, dtype)
    if dtype == "f16":
        assert torch.equal(out.cpu(), torch.from_numpy(ref))
    else:
        assert np.array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)
    if shape[0] % 64 == 0 and shape[1] % 64 == 0:
        out_t = ops.nf4_dequant(_W(st), transpose=True, dtype=tdt)
        assert torch.equal(out_t.cpu(), out.cpu().t().contiguous())


def test_nf4_dequant_nested_segments():
    """Three weights back to back (q, k, v): only the double-quantisation offset differs per
    segment (solution/engine.py:112-157)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    rng = np.random.default_rng(5)
    parts = [quantize_nf4((rng.standard_normal((r, 256)) * 0.03).astype(np.float32), nested=True)
             for r in (256, 128, 128)]

    class St:
        pass

    st = St()
    st.shape = (512, 256)
    st.packed = np.concatenate([p.packed for p in parts])
    st.absmax = np.concatenate([p.absmax for p in parts])
    st.absmax2 = np.concatenate([p.absmax2 for p in parts])
    st.code2 = parts[0].code2
    st.code = parts[0].code
    st.nested, st.bs2 = True, 256
    st.offset = parts[0].offset
    offsets = np.concatenate([p.offset for p in parts])
    seg1 = 256 * 256 // 64
    seg2 = seg1 + 128 * 256 // 64
    out = ops.nf4_dequant(_W(st, seg1, seg2, offsets))
    ref = np.concatenate([dequant_nf4(p) for p in parts])
    assert torch.equal(out.cpu(), torch.from_numpy(ref))


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (37, 256, 1536), (300, 2048, 1536),
                                   (1400, 17920, 1536), (1400, 1536, 8960), (129, 200, 136),
                                   (1000, 151936 // 8, 1536), (1090, 1536, 1536),
                                   (1090, 8960, 1536), (1090, 17920, 1536), (200, 96, 512),
                                   (1090, 1536, 17920)])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_matches_torch(M, N, K, dt):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(M * 31 + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(dt)
    b = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(dt)
    bias = torch.randn(N, device=DEV, generator=g).to(dt)
    ref = a.float() @ b.float().t()
    out = ops.gemm(a, b)
    tol = 2e-2 if dt == torch.bfloat16 else 4e-3
    scale = ref.abs().max().item() + 1e-6
    assert (out.float() - ref).abs().max().item() / scale < tol
    out32 = ops.gemm(a, b, out_dtype=torch.float32, bias=bias)
    assert (out32 - (ref + bias.float())).abs().max().item() / scale < 1e-3
    ops.gemm(a, b, out=out32, accumulate=True)
    assert (out32 - (2 * ref + bias.float())).abs().max().item() / scale < 2e-3
    assert ops.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1090, 8960, 1536), (1090, 1536, 17920), (1090, 1536, 1536),
                                   (1090, 1536, 2048), (37, 192, 64), (129, 200, 136),
                                   (300, 96, 512), (1, 8, 8)])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_nn_matches_torch(M, N, K, dt):
    """C = A . B with B stored [K, N] (the forward-layout weight in the data-gradient products),
    read as an MN-major tensor-core operand."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(dt)
    b = (torch.randn(K, N, device=DEV, generator=g) * 0.05).to(dt)
    ref = a.float() @ b.float()
    out = ops.gemm(a, b, b_kn=True)
    tol = 2e-2 if dt == torch.bfloat16 else 4e-3
    scale = ref.abs().max().item() + 1e-6
    assert (out.float() - ref).abs().max().item() / scale < tol
    res = torch.randn(M, N, device=DEV, generator=g)
    out32 = ops.gemm(a, b, b_kn=True, out_dtype=torch.float32, residual=res)
    assert (out32 - (res + out.float())).abs().max().item() / scale < 2e-3
    assert ops.device_status() == 0


@pytest.mark.parametrize("M,N,K,b_kn", [(256, 256, 128, False), (1090, 1536, 1536, False),
                                        (1090, 17920, 1536, False), (1090, 8960, 1536, False),
                                        (37, 200, 64, False), (1000, 151936 // 8, 1536, False),
                                        (1090, 1536, 8960, True), (1090, 1536, 17920, True),
                                        (129, 128, 136, True), (300, 8960, 1536, True)])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_pair_tiles(M, N, K, b_kn, dt):
    """The 2-SM path (256-row pair tiles over a CTA pair, tcgen05 cta_group::2) forced on for
    every shape: against torch, with the residual epilogue, and bit-equal on a second call."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(M * 5 + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(dt)
    b = (torch.randn(*((K, N) if b_kn else (N, K)), device=DEV, generator=g) * 0.05).to(dt)
    ref = a.float() @ (b.float() if b_kn else b.float().t())
    res = torch.randn(M, N, device=DEV, generator=g)
    ops.gemm_set_mode(2)
    try:
        out = ops.gemm(a, b, b_kn=b_kn)
        again = ops.gemm(a, b, b_kn=b_kn)
        out32 = ops.gemm(a, b, b_kn=b_kn, out_dtype=torch.float32, residual=res)
    finally:
        ops.gemm_set_mode(0)
    tol = 2e-2 if dt == torch.bfloat16 else 4e-3
    scale = ref.abs().max().item() + 1e-6
    assert (out.float() - ref).abs().max().item() / scale < tol
    assert torch.equal(out, again)
    assert (out32 - (res + out.float())).abs().max().item() / scale < 2e-3
    assert ops.device_status() == 0


@pytest.mark.parametrize("N,K,M", [(2048, 1536, 1090), (1536, 1536, 300), (17920, 1536, 1090),
                                   (1536, 8960, 1090), (200, 128, 37), (256, 64, 1)])
@pytest.mark.parametrize("nested", [False, True])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_nf4_fused_equals_dequant_then_gemm(N, K, M, nested, dt):
    """The NF4-fused GEMM in both layouts against ql_nf4_dequant + the dense GEMM on the same
    bytes (the same 16-bit weight, the same fp32 accumulation order), and against torch."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    g = torch.Generator().manual_seed(N + K + M + int(nested))
    st = quantize_nf4(np.asarray(torch.randn(N, K, generator=g) * 0.05), nested=nested)
    w = _W(st)
    W = ops.nf4_dequant(w, dtype=dt)  # [N, K]
    a = torch.randn(M, K, device=DEV, generator=torch.Generator(device=DEV).manual_seed(M)).to(dt)
    bias = torch.randn(N, device=DEV).to(dt)
    fused = ops.gemm_nf4(a, w, layout=0, bias=bias)
    dense = ops.gemm(a, W, bias=bias)
    ref = a.float() @ W.float().t() + bias.float()
    scale = ref.abs().max().item() + 1e-6
    tol = 2e-2 if dt == torch.bfloat16 else 4e-3
    assert (fused.float() - ref).abs().max().item() / scale < tol
    ulp = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10  # one rounding step of the output
    assert (fused.float() - dense.float()).abs().max().item() / scale <= ulp
    res = torch.randn(M, N, device=DEV)
    f32 = ops.gemm_nf4(a, w, layout=0, out_dtype=torch.float32, residual=res)
    plain = ops.gemm_nf4(a, w, layout=0)  # residual epilogue: res + round16(A W^T)
    assert (f32 - (res + plain.float())).abs().max().item() / scale < 1e-5
    if N % 64 == 0:  # layout 1: dX[M, K] = dY[M, N] . W[N, K]
        dy = torch.randn(M, N, device=DEV).to(dt)
        dx = ops.gemm_nf4(dy, w, layout=1)
        ref1 = dy.float() @ W.float()
        s1 = ref1.abs().max().item() + 1e-6
        assert (dx.float() - ref1).abs().max().item() / s1 < tol
        assert (dx.float() - ops.gemm(dy, W, b_kn=True).float()).abs().max().item() / s1 <= ulp
    assert ops.device_status() == 0


def test_nf4_dequant_batch_equals_per_weight_dequant():
    """ql_nf4_dequant_batch over 31 weights (two launches, plain and nested scales) equals
    ql_nf4_dequant of each, bit for bit."""
    import ctypes

    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib, ops

    g = torch.Generator().manual_seed(3)
    shapes = [(64 * (1 + i % 5), 64 * (1 + i % 3)) for i in range(31)]
    ws = [_W(quantize_nf4(np.asarray(torch.randn(r, c, generator=g) * 0.1), nested=bool(i % 2)))
          for i, (r, c) in enumerate(shapes)]
    for dt in (torch.float16, torch.bfloat16):
        outs = [torch.full(w.shape, float("nan"), device=DEV, dtype=dt) for w in ws]
        arr = (_lib.STRUCTS["ql_nf4_weight"] * len(ws))(*[ops.nf4_weight_struct(w) for w in ws])
        ptrs = (ctypes.c_void_p * len(ws))(*[o.data_ptr() for o in outs])
        _lib.call("ql_nf4_dequant_batch", ctypes.addressof(arr), ctypes.addressof(ptrs), len(ws),
                  ops.dtype_code(dt), torch.cuda.current_stream().cuda_stream)
        for w, o in zip(ws, outs):
            assert torch.equal(o, ops.nf4_dequant(w, dtype=dt))
    assert ops.device_status() == 0


def test_gemm_strided_output():
    """C written into columns of a wider buffer (the [gate | up] halves, the LoRA slices)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    a = torch.randn(200, 512, device=DEV).half()
    b = torch.randn(256, 512, device=DEV).half() * 0.05
    buf = torch.zeros(200, 1024, device=DEV, dtype=torch.half)
    ops.gemm(a, b, out=buf[:, 512:768])
    ref = a.float() @ b.float().t()
    assert (buf[:, 512:768].float() - ref).abs().max() < 2e-2 * ref.abs().max()
    assert buf[:, :512].abs().max() == 0 and buf[:, 768:].abs().max() == 0


def test_bf16_helpers():
    x = np.array([1.0, 1.00390625, -3.5, 1e-3], np.float32)
    from oracle.nf4 import f32_to_bf16_bits

    back = bf16_bits_to_f32(f32_to_bf16_bits(x))
    assert np.allclose(back, torch.tensor(x).bfloat16().float().numpy())


@pytest.mark.parametrize("M,N,K", [(300, 256, 17920), (130, 1536, 8960), (1090, 512, 8960),
                                   (64, 1536, 17920)])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_split_k(M, N, K, dt):
    """Shapes with too few output tiles to fill the GPU split K; the partial sums are added in a
    fixed order, so two calls agree bit for bit, and the result matches the unsplit GEMM (no
    workspace) to rounding. Split-K belongs to the single-CTA tiles: those are forced here."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    ops.gemm_set_mode(1)
    try:
        _split_k_case(M, N, K, dt)
    finally:
        ops.gemm_set_mode(0)


def _split_k_case(M, N, K, dt):
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib, ops

    assert _lib.lib().ql_gemm_workspace_bytes(M, N, K) > 0
    g = torch.Generator(device=DEV).manual_seed(M + 7 * N + K)
    a = torch.randn(M, K, device=DEV, generator=g).to(dt)
    b = (torch.randn(N, K, device=DEV, generator=g) * 0.05).to(dt)
    res = torch.randn(M, N, device=DEV, generator=g)
    ref = a.float() @ b.float().t()
    scale = ref.abs().max().item()
    out1 = ops.gemm(a, b)
    out2 = ops.gemm(a, b)
    assert torch.equal(out1, out2)
    tol = 2e-2 if dt == torch.bfloat16 else 4e-3
    assert (out1.float() - ref).abs().max().item() / scale < tol
    # residual epilogue: C = residual + round16(A B^T)
    out32 = ops.gemm(a, b, out_dtype=torch.float32, residual=res)
    assert (out32 - (res + out1.float())).abs().max().item() / scale < 2e-3
    # the same GEMM with no workspace runs unsplit
    plain = torch.empty(M, N, device=DEV, dtype=dt)
    _lib.call("ql_gemm_tn", a.data_ptr(), K, b.data_ptr(), K, plain.data_ptr(), N, None, M, N, K,
              ops.dtype_code(dt), ops.dtype_code(dt), 0, None, None, 0,
              torch.cuda.current_stream().cuda_stream)
    assert (plain.float() - out1.float()).abs().max().item() / scale < tol
    ws = ops.gemm_workspace(a.device, 2048)
    assert int(ws[:2048].count_nonzero()) == 0  # the tile counters are left at zero
    assert ops.device_status() == 0



@pytest.mark.parametrize("M,N,K,b_kn", [(1090, 2048, 1536, False), (1090, 17920, 1536, False),
                                        (1090, 1536, 1536, True), (300, 8960, 1536, True),
                                        (777, 256, 384, False), (2100, 1536, 2048, True)])
@pytest.mark.parametrize("tiles", [0, 1, 2])
def test_gemm_two_chunk_stages_equal_single_chunk(M, N, K, b_kn, tiles):
    """Pipeline stages of two 64-wide K chunks (one 3-D copy per operand: the default for
    single-CTA tiles of up to 128 columns where K is a multiple of 128) and of one chunk (2-D
    copies, mode bit 4) issue the same MMAs in the same K order, so without split-K (K <= 2048
    here) the outputs are equal; every tile-kind mode (cost model, single-CTA, 2-SM pairs, which
    keep one-chunk stages)."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    a = torch.randn(M, K, device=DEV, generator=g).half()
    b = (torch.randn(K, N, device=DEV, generator=g) * 0.05).half() if b_kn else \
        (torch.randn(N, K, device=DEV, generator=g) * 0.05).half()
    try:
        ops.gemm_set_mode(tiles)
        two = ops.gemm(a, b, b_kn=b_kn)
        ops.gemm_set_mode(tiles + 4)
        one = ops.gemm(a, b, b_kn=b_kn)
    finally:
        ops.gemm_set_mode(0)
    assert torch.equal(two, one)
    ref = a.float() @ (b.float() if b_kn else b.float().t())
    assert (two.float() - ref).abs().max().item() / (ref.abs().max().item() + 1e-6) < 4e-3
    assert ops.device_status() == 0

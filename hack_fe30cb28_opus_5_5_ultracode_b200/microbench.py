"""Per-kernel timing of the fused step's kernels at the Qwen2.5-1.5B shapes, with CUDA events
on the launching stream (warm-up, then `--iters` launches, each input set larger than L2):

    python -m hack_fe30cb28_opus_5_5_ultracode_b200.microbench [--tokens 1090] [--iters 20]
        [--only gemm|dequant|attn|rms|glu|rope|ce|head]

Prints one JSON line per kernel and shape: average launch time, algorithmic FLOPs or bytes per
launch, achieved TFLOP/s or GB/s and the fraction of the measured peak (MEASURED_PEAKS.json).
The layer GEMMs are also timed through cuBLAS (`torch.mm`, lines "cublas ...") for comparison.
Also the small, self-contained case the ncu captures run on.
"""

import argparse
import json
import os

import torch

from . import ops
from .model import QWEN25_1P5B, quantize_nf4

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return p["hbm_gbs"], p["bf16_tflops"]
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0


def _time(fn, iters):
    """Seconds per launch of fn, the launches replayed from a CUDA graph (no host overhead
    between them)."""
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn(0)  # (warm-up on the capture stream)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(iters):
                fn(i)
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters / 1e3


def _report(name, shape, sec, flops=None, nbytes=None):
    hbm, tf = _peaks()
    line = {"kernel": name, "shape": shape, "us": sec * 1e6}
    if flops:
        line.update(tflops=flops / sec / 1e12, frac_of_measured_bf16=flops / sec / 1e12 / tf)
    if nbytes:
        line.update(gbs=nbytes / sec / 1e9, frac_of_measured_hbm=nbytes / sec / 1e9 / hbm)
    print(json.dumps(line), flush=True)


class _W:
    def __init__(self, p):
        qs = p.quant_state
        self.shape = tuple(qs.shape)
        self.packed = p.data.reshape(-1)
        self.absmax = qs.absmax
        self.code = qs.code
        self.nested, self.bs2 = False, 1
        self.code2 = self.absmax2 = self.offsets = None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=1090)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--gemm-mode", type=int, default=0,
                    help="GEMM tile kind: 0 cost model, 1 single-CTA, 2 2-SM pair tiles")
    ap.add_argument("--only", default=None,
                    help="gemm | gemm:<qkv|o|gate_up|down|lm_head> | dequant | attn | glu | rms | ce")
    args = ap.parse_args()
    dev = torch.device("cuda")
    ops.gemm_set_mode(args.gemm_mode)
    cfg = QWEN25_1P5B
    n, H, I, V = args.tokens, cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    HQ, HKV, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    dt = torch.float16
    g = torch.Generator(device=dev).manual_seed(0)
    only = args.only.split(":")[0] if args.only else None
    shape_only = args.only.split(":")[1] if args.only and ":" in args.only else None
    want = (lambda k: only is None or only == k)
    want_shape = (lambda name: shape_only is None or shape_only == name)
    copies = 4  # rotate inputs so consecutive launches do not hit L2

    if want("gemm") or want("dequant"):
        shapes = {"qkv": ((HQ + 2 * HKV) * D, H), "o": (H, HQ * D), "gate_up": (2 * I, H),
                  "down": (H, I)}
        for name, (N, K) in shapes.items():
            if not want_shape(name):
                continue
            ws = [_W(quantize_nf4(torch.randn(N, K, device=dev, generator=g) * 0.02))
                  for _ in range(2)]
            if want("dequant"):
                outs = [torch.empty(N, K, device=dev, dtype=dt) for _ in range(2)]
                nbytes = N * K * (0.5 + 4 / 64 + 2)
                sec = _time(lambda i: ops.nf4_dequant(ws[i % 2], out=outs[i % 2]), args.iters)
                _report("nf4_dequant", [N, K], sec, nbytes=nbytes)
                sec = _time(lambda i: ops.nf4_dequant(ws[i % 2], out=outs[i % 2].view(K, N),
                                                      transpose=True), args.iters)
                _report("nf4_dequant_t", [K, N], sec, nbytes=nbytes)
            if want("gemm"):
                a = [torch.randn(n, K, device=dev, generator=g).to(dt) for _ in range(copies)]
                b = [torch.randn(N, K, device=dev, generator=g).to(dt) * 0.02 for _ in range(2)]
                c = [torch.empty(n, N, device=dev, dtype=dt) for _ in range(copies)]
                sec = _time(lambda i: ops.gemm(a[i % copies], b[i % 2], out=c[i % copies]),
                            args.iters)
                _report("gemm_tn " + name, [n, N, K], sec, flops=2.0 * n * N * K)
                # cuBLAS on the same operands, for comparison (torch.mm)
                sec = _time(lambda i: torch.mm(a[i % copies], b[i % 2].t(), out=c[i % copies]),
                            args.iters)
                _report("cublas " + name, [n, N, K], sec, flops=2.0 * n * N * K)
                # the data-gradient GEMM of the same projection: [n, N] x [K, N]^T
                at = [torch.randn(n, N, device=dev, generator=g).to(dt) for _ in range(copies)]
                bt = [torch.randn(K, N, device=dev, generator=g).to(dt) * 0.02 for _ in range(2)]
                ct = [torch.empty(n, K, device=dev, dtype=dt) for _ in range(copies)]
                sec = _time(lambda i: ops.gemm(at[i % copies], bt[i % 2], out=ct[i % copies]),
                            args.iters)
                _report("gemm_tn dgrad " + name, [n, K, N], sec, flops=2.0 * n * N * K)
                sec = _time(lambda i: torch.mm(at[i % copies], bt[i % 2].t(), out=ct[i % copies]),
                            args.iters)
                _report("cublas dgrad " + name, [n, K, N], sec, flops=2.0 * n * N * K)
                # NF4 dequantised inside the GEMM (no 16-bit weight in HBM), both layouts
                sec = _time(lambda i: ops.gemm_nf4(a[i % copies], ws[i % 2], layout=0,
                                                   out=c[i % copies]), args.iters)
                _report("gemm_nf4 " + name, [n, N, K], sec, flops=2.0 * n * N * K)
                if K % 64 == 0 and N % 64 == 0:
                    sec = _time(lambda i: ops.gemm_nf4(at[i % copies], ws[i % 2], layout=1,
                                                       out=ct[i % copies]), args.iters)
                    _report("gemm_nf4 dgrad " + name, [n, K, N], sec, flops=2.0 * n * N * K)
                # the same product straight from the forward-layout weight (MN-major B)
                sec = _time(lambda i: ops.gemm(at[i % copies], b[i % 2], out=ct[i % copies],
                                               b_kn=True), args.iters)
                _report("gemm_nn dgrad " + name, [n, K, N], sec, flops=2.0 * n * N * K)
    if want("gemm") and want_shape("lm_head"):
        hn = torch.randn(n, H, device=dev, generator=g).to(dt)
        W = torch.randn(V, H, device=dev, generator=g).to(dt) * 0.02
        logits = torch.empty(n, V, device=dev, dtype=dt)
        sec = _time(lambda i: ops.gemm(hn, W, out=logits), args.iters)
        _report("gemm_tn lm_head", [n, V, H], sec, flops=2.0 * n * V * H)
        WT = W.t().contiguous()
        sec = _time(lambda i: ops.gemm(logits, WT), args.iters)
        _report("gemm_tn lm_head dgrad", [n, H, V], sec, flops=2.0 * n * V * H)
        sec = _time(lambda i: ops.gemm(logits, W, b_kn=True), args.iters)
        _report("gemm_nn lm_head dgrad", [n, H, V], sec, flops=2.0 * n * V * H)
    if want("attn"):
        # the bench's short packed sequences, or (attn:long) configs[2]-like long ones
        lengths = [3072, 2560, 4096, 2048] if shape_only == "long" else [300, 257, 400, 133]
        m = sum(lengths)
        cu = torch.tensor([0] + torch.tensor(lengths).cumsum(0).tolist(), device=dev,
                          dtype=torch.int32)
        q = torch.randn(m, HQ, D, device=dev, generator=g).to(dt)
        k = torch.randn(m, HKV, D, device=dev, generator=g).to(dt)
        v = torch.randn(m, HKV, D, device=dev, generator=g).to(dt)
        flops = sum(4.0 * L * (L + 1) / 2 * HQ * D for L in lengths)
        out, lse = ops.attn_fwd(q, k, v, cu, max(lengths), D ** -0.5)
        for impl, name in ((1, "attn_fwd mma.sync"), (0, "attn_fwd")):
            ops.attn_set_impl(impl)
            sec = _time(lambda i: ops.attn_fwd(q, k, v, cu, max(lengths), D ** -0.5, out=out,
                                               lse=lse), args.iters)
            _report(name, lengths, sec, flops=flops)
        dout = torch.randn_like(q)
        for impl, name in ((1, "attn_bwd mma.sync"), (0, "attn_bwd")):
            ops.attn_set_impl(impl)
            sec = _time(lambda i: ops.attn_bwd(dout, q, k, v, out, lse, cu, max(lengths),
                                               D ** -0.5), args.iters)
            _report(name, lengths, sec, flops=2.5 * flops)
    if want("glu"):
        gu = [torch.randn(n, 2 * I, device=dev, generator=g).to(dt) for _ in range(copies)]
        m_ = [torch.empty(n, I, device=dev, dtype=dt) for _ in range(copies)]
        sec = _time(lambda i: ops.glu_fwd(gu[i % copies], I, out=m_[i % copies]), args.iters)
        _report("glu_fwd", [n, I], sec, nbytes=n * I * 6)
        sec = _time(lambda i: ops.glu_bwd(m_[i % copies], gu[i % copies], I), args.iters)
        _report("glu_bwd", [n, I], sec, nbytes=n * I * 10)
    if want("rms"):
        xs = [torch.randn(n, H, device=dev, generator=g) for _ in range(copies)]
        w = torch.ones(H, device=dev)
        A = torch.randn(16, H, device=dev, generator=g).to(dt) * 0.02
        tok = torch.arange(n, device=dev)
        drop = ops.Drop(tok, 1, 0, 10, 1184 * 256, 0.05)
        ys = [torch.empty(n, H, device=dev, dtype=dt) for _ in range(copies)]
        sec = _time(lambda i: ops.rms_fwd(xs[i % copies], w, 1e-6, drop=drop, Aq=A, Av=A,
                                          want_yq=True, out_y=ys[i % copies]), args.iters)
        _report("rms_fwd (+dropout, LoRA-A)", [n, H], sec, nbytes=n * H * (4 + 3 * 2))
        sec = _time(lambda i: ops.rms_fwd(xs[i % copies], w, 1e-6, out_y=ys[i % copies]),
                    args.iters)
        _report("rms_fwd (plain)", [n, H], sec, nbytes=n * H * (4 + 2))
        rstd = torch.ones(n, device=dev)
        dy = [torch.randn(n, H, device=dev, generator=g).to(dt) for _ in range(copies)]
        lo = torch.randn(n, 16, device=dev, generator=g)
        dx = [torch.empty(n, H, device=dev) for _ in range(copies)]
        sec = _time(lambda i: ops.rms_bwd(dy[i % copies], xs[i % copies], rstd, w, dres=xs[0],
                                          dxlo_q=lo, dxlo_v=lo, Aq=A, Av=A, drop=drop,
                                          out=dx[i % copies]), args.iters)
        _report("rms_bwd (+dropout, LoRA dx)", [n, H], sec, nbytes=n * H * (2 + 4 + 4 + 4))
    if want("rope"):
        C = (HQ + 2 * HKV) * D
        qkv = [torch.randn(n, C, device=dev, generator=g).to(dt) for _ in range(copies)]
        xq = torch.randn(n, 16, device=dev, generator=g).to(dt)
        Bq = torch.randn(HQ * D, 16, device=dev, generator=g).to(dt) * 0.02
        Bv = torch.randn(HKV * D, 16, device=dev, generator=g).to(dt) * 0.02
        pos = torch.arange(n, device=dev, dtype=torch.int32) % 512
        cos = torch.rand(1024, D // 2, device=dev)
        sin = torch.rand(1024, D // 2, device=dev)
        outs = [(torch.empty(n, HQ, D, device=dev, dtype=dt), torch.empty(n, HKV, D, device=dev, dtype=dt),
                 torch.empty(n, HKV, D, device=dev, dtype=dt)) for _ in range(copies)]
        sec = _time(lambda i: ops.rope_fwd(qkv[i % copies], cos, sin, pos, HQ, HKV, D, 2.0, xq=xq,
                                           xv=xq, Bq=Bq, Bv=Bv, out=outs[i % copies]), args.iters)
        _report("rope_fwd (+LoRA-B)", [n, C], sec, nbytes=n * C * 4)
        dq = torch.randn(n, HQ, D, device=dev, generator=g)
        dk = torch.randn(n, HKV, D, device=dev, generator=g)
        sec = _time(lambda i: ops.rope_bwd(dq, dk, dk, cos, sin, pos, HQ, HKV, D, Bq=Bq, Bv=Bv,
                                           lora_scale=2.0, out=qkv[i % copies]), args.iters)
        _report("rope_bwd (+LoRA dx)", [n, C], sec, nbytes=n * C * 6)
    if want("colsum"):
        X = torch.randn(n, H, device=dev, generator=g).to(dt)
        Y = torch.randn(n, 16, device=dev, generator=g)
        out = torch.empty(16, H, device=dev)
        ws = torch.empty(64 * H * 16, device=dev)
        sec = _time(lambda i: ops.lora_colsum(X, Y, transpose=True, out=out, workspace=ws),
                    args.iters)
        _report("lora_colsum", [n, H], sec, nbytes=n * H * 2)
        # the four products of a layer in one launch (what the layer backward runs)
        C = (HQ + 2 * HKV) * D
        gq = torch.randn(n, C, device=dev, generator=g).to(dt)
        x16 = Y.to(dt)
        jobs = [(gq[:, :HQ * D], x16, 2.0, False), (gq[:, (HQ + HKV) * D:], x16, 2.0, False),
                (X, Y, 1.0, True), (X, Y, 1.0, True)]
        sec = _time(lambda i: ops.lora_grads(jobs), args.iters)
        _report("lora_grads (4 products)", [n, (HQ + HKV) * D + 2 * H], sec,
                nbytes=n * ((HQ + HKV) * D + 2 * H) * 2)
    if want("head"):
        # the head over a block of rows (70 % with a target): the chunked, L2-resident form the
        # step runs (VocabHead) against materialised [rows, V] logits (logits GEMM, ce_rows,
        # data-gradient GEMM), same inputs
        from .engine import VocabHead

        W = (torch.randn(V, H, device=dev, generator=g) * 0.02).to(dt)
        hn = torch.randn(n, H, device=dev, generator=g).to(dt)
        sup = int(0.7 * n)
        tgt = torch.randint(0, V, (n,), device=dev, generator=g)
        tgt[sup:] = -100
        stats = [torch.empty(n, device=dev), torch.empty(n, device=dev),
                 torch.empty(n, device=dev, dtype=torch.int32)]
        head = VocabHead(W, dt)
        flops = 2.0 * V * H * (n + sup)
        sec = _time(lambda i: head.block(hn, tgt, sup, *stats), args.iters)
        _report(f"head chunked ({head.chunk_width(n)}-entry chunks)", [n, V, H], sec, flops=flops)
        logits = torch.empty(n, V, device=dev, dtype=dt)

        def materialised(i):
            ops.gemm(hn, W, out=logits)
            ops.ce_rows(logits, tgt, write_grad=True, loss=stats[0], entropy=stats[1],
                        correct=stats[2])
            ops.gemm(logits[:sup], W, b_kn=True)

        sec = _time(materialised, args.iters)
        _report("head materialised logits", [n, V, H], sec, flops=flops)
    if want("ce"):
        logits = [torch.randn(n, V, device=dev, generator=g).to(dt) for _ in range(2)]
        tgt = torch.randint(0, V, (n,), device=dev, generator=g)
        sec = _time(lambda i: ops.ce_rows(logits[i % 2], tgt), args.iters)
        _report("ce_rows", [n, V], sec, nbytes=n * V * 2 * 3)


if __name__ == "__main__":
    main()

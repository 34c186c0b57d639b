"""Generates the golden fixtures in this folder from the reference's OWN Triton kernels, run on
CPU tensors under TRITON_INTERPRET=1 (only where the reference tree is mounted: the build
container; nothing on the GPU box reads the reference).

    python tests/golden/make_golden.py /path/to/the/reference/checkout

Each fixture holds seeded inputs and the reference kernel's outputs:
  nf4.npz        nf4_dequant_kernel (non-nested; the interpreter lacks libdevice.mul_rn for
                 the nested path, which is pinned against the oracle's formula instead)
  dropout.npz    torch_dropout_keep_kernel for several (seed, counter, threads, p, VEC)
  rms.npz        rms_fwd_kernel (residual add, both LoRA dropouts) and rms_bwd_kernel
  rope.npz       qkv_rope_fwd_kernel / qkv_rope_bwd_kernel (HQ 12, HKV 2, D 128)
  glu.npz        glu_fwd_kernel / glu_bwd_kernel
  ce.npz         lm_head_ce_kernel, lm_head_piece_kernel + lm_head_finish_kernel
"""

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_golden.py /path/to/the/reference/checkout")
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from solution import kernels as K  # noqa: E402  (the reference's kernels)

from oracle.nf4 import quantize_nf4  # noqa: E402


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **{k: (v.numpy() if torch.is_tensor(v) else np.asarray(v))
                                 for k, v in arrays.items()})
    print("wrote", path, sum(np.asarray(v).nbytes for v in arrays.values()), "bytes")


def gen_nf4():
    rng = np.random.default_rng(0)
    rows, cols = 192, 256
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    st = quantize_nf4(w)
    blocks = rows * cols // 64
    out = torch.empty((rows, cols), dtype=torch.float16)
    absmax = torch.from_numpy(st.absmax)
    K.nf4_dequant_kernel[(-(-blocks // 32),)](
        torch.from_numpy(st.packed), absmax, absmax, absmax, absmax,
        torch.from_numpy(st.code), out, blocks, NESTED=False, STANDARD_NF4=True, BS1=64, BS2=1,
        ROWS=32)
    save("nf4.npz", packed=st.packed, absmax=st.absmax, rows=rows, cols=cols, out=out)


def gen_dropout():
    cases = [(1234, 0, 1184 * 256, 0.05, 4, 4096), (987654321, 17, 40 * 4 * 256, 0.1, 4, 5000),
             (-3, 5, 256, 0.25, 4, 3000), (42, 100, 1184 * 256, 0.1, 8, 8192)]
    out = {}
    for i, (seed, ctr, G, p, vec, n) in enumerate(cases):
        m = torch.empty(n, dtype=torch.int8)
        K.torch_dropout_keep_kernel[(-(-n // 1024),)](m, n, seed, ctr, G, 1.0 - p, VEC=vec,
                                                      BLOCK=1024)
        out[f"case{i}"] = np.array([seed, ctr, G, vec, n], np.int64)
        out[f"p{i}"] = np.float64(p)
        out[f"keep{i}"] = m.numpy()
    save("dropout.npz", **out)


def gen_rms():
    g = torch.Generator().manual_seed(1)
    n, H = 9, 256
    x = torch.randn(n, H, generator=g) * 3
    delta = torch.randn(n, H, generator=g).to(torch.float16)
    w = torch.rand(H, generator=g) + 0.5
    tok = (torch.arange(n) * 3 + 1).to(torch.int64)
    p = 0.25
    seed, ctr_q, ctr_v, G = 77, 11, 12, 1184 * 256
    xsum = torch.empty_like(x)
    y = torch.empty(n, H, dtype=torch.float16)
    yq = torch.empty_like(y)
    yv = torch.empty_like(y)
    rstd = torch.empty(n)
    K.rms_fwd_kernel[(n,)](x, delta, w, xsum, y, yq, yv, rstd, tok, H, 1e-6, 1 - p, 1 / (1 - p),
                           seed, ctr_q, ctr_v, G, 1, 1, 1, 1, VEC=4, BLOCK=H)
    dy = torch.randn(n, H, generator=g).to(torch.float16)
    tq = torch.randn(n, H, generator=g).to(torch.float16)
    tv = torch.randn(n, H, generator=g).to(torch.float16)
    dres = torch.randn(n, H, generator=g)
    dx = torch.empty_like(x)
    K.rms_bwd_kernel[(n,)](dy, tq, tv, xsum, rstd, w, dres, dx, tok, H, H, 1 - p, 1 / (1 - p),
                           seed, ctr_q, ctr_v, G, 0.5, 1, 1, 1, VEC=4, BLOCK=H)
    save("rms.npz", x=x, delta=delta, w=w, tok=tok, p=p, seed=seed, ctr_q=ctr_q, ctr_v=ctr_v,
         G=G, eps=1e-6, xsum=xsum, y=y, yq=yq, yv=yv, rstd=rstd, dy=dy, tq=tq, tv=tv, dres=dres,
         grad_scale=0.5, dx=dx)


def gen_rope():
    g = torch.Generator().manual_seed(2)
    n, HQ, HKV, D = 7, 12, 2, 128
    C = (HQ + 2 * HKV) * D
    qkv = torch.randn(n, C, generator=g).to(torch.float16)
    lq = torch.randn(n, HQ * D, generator=g).to(torch.float16)
    lv = torch.randn(n, HKV * D, generator=g).to(torch.float16)
    pos = torch.randint(0, 300, (n,), generator=g, dtype=torch.int32)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2).float() / D))
    freqs = torch.arange(512).float()[:, None] * inv[None, :]
    cos, sin = freqs.cos().contiguous(), freqs.sin().contiguous()
    q = torch.empty(n, HQ, D, dtype=torch.float16)
    k = torch.empty(n, HQ, D, dtype=torch.float16)
    v = torch.empty(n, HQ, D, dtype=torch.float16)
    K.qkv_rope_fwd_kernel[(n,)](qkv, lq, lv, cos, sin, pos, q, k, v, 2.0, HQ=HQ, HKV=HKV, D=D,
                                BHQ=16, BHKV=2, GROUP=HQ // HKV, LORA_Q=True, LORA_V=True)
    dq = torch.randn(n, HQ, D, generator=g).to(torch.float16)
    dk = torch.randn(n, HQ, D, generator=g).to(torch.float16)
    dv = torch.randn(n, HQ, D, generator=g).to(torch.float16)
    dqkv = torch.empty(n, C, dtype=torch.float16)
    K.qkv_rope_bwd_kernel[(n,)](dq, dk, dv, cos, sin, pos, dqkv, HQ=HQ, HKV=HKV, D=D, BHQ=16,
                                BHKV=2, GROUP=HQ // HKV)
    save("rope.npz", qkv=qkv, lq=lq, lv=lv, pos=pos, cos=cos, sin=sin, scale=2.0, q=q, k=k, v=v,
         dq=dq, dk=dk, dv=dv, dqkv=dqkv)


def gen_glu():
    g = torch.Generator().manual_seed(3)
    n, I = 5, 1000
    gu = (torch.randn(n, 2 * I, generator=g) * 3).to(torch.float16)
    m = torch.empty(n, I, dtype=torch.float16)
    K.glu_fwd_kernel[(n, 1)](gu, m, I, BLOCK=1024)
    dm = torch.randn(n, I, generator=g).to(torch.float16)
    gu_in = gu.clone()
    K.glu_bwd_kernel[(n, 1)](dm, gu, I, BLOCK=1024)
    save("glu.npz", gu=gu_in, m=m, dm=dm, dgu=gu)


def gen_ce():
    g = torch.Generator().manual_seed(4)
    n, V, H = 6, 5000, 64
    logits = (torch.randn(n, V, generator=g) * 4).to(torch.float16)
    target = torch.randint(0, V, (n,), generator=g)
    target[2] = -100
    target[1] = int(logits[1].float().argmax())
    work = logits.clone()
    loss = torch.empty(n)
    ent = torch.empty(n)
    correct = torch.empty(n, dtype=torch.int32)
    K.lm_head_ce_kernel[(n,)](work, target, loss, ent, correct, V, 1, BLOCK=4096)
    save("ce.npz", logits=logits, target=target, loss=loss, entropy=ent, correct=correct,
         grad=work)


if __name__ == "__main__":
    torch.set_num_threads(4)
    gen_nf4()
    gen_dropout()
    gen_rms()
    gen_rope()
    gen_glu()
    gen_ce()

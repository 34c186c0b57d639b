"""CPU oracle of the fused QLoRA step — TEST INFRASTRUCTURE ONLY.

A plain numpy / torch-CPU restatement of the reference's algorithm for the hot path
(Magurin/hack-fe30cb28-opus-5-5-ultracode, solution/kernels.py and solution/engine.py), each
function citing the reference lines it follows. Only tests/, __graft_entry__.smoke() and the
cpu_baseline / reference arm of bench.py may import it, and only as the checker or the timed CPU
baseline: the product path (the package hack_fe30cb28_opus_5_5_ultracode_b200) never calls it and
fails loudly when its CUDA library is missing.

Pinning: the elementwise pieces (NF4 dequant, the PyTorch-dropout Philox mask, RMSNorm fwd/bwd,
qkv+RoPE fwd/bwd, SwiGLU fwd/bwd, the cross-entropy head kernels) are checked against golden
vectors produced by the reference's own Triton kernels run under TRITON_INTERPRET=1 in the
build container (tests/golden/make_golden.py, fixtures in tests/golden/). NF4 *quantisation*
(bitsandbytes, absent here) is parity-unpinned: the quantiser below only has to produce valid
NF4 bytes, the dequantisation formula is what the hot path must reproduce bit for bit.
"""

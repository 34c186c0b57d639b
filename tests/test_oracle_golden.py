"""CPU: the oracle against the golden fixtures of the reference's own kernels (pins the oracle
that the GPU parity tests then hold the CUDA kernels to)."""

import numpy as np

from oracle import kernels as OK
from oracle.nf4 import NF4_LEVELS, QuantState, dequant_nf4, quantize_nf4
from oracle.philox import dropout_keep, draw, philox4x32_10


def test_nf4_dequant_bit_exact_vs_reference(golden):
    g = golden("nf4.npz")
    st = QuantState(g["packed"], g["absmax"], (int(g["rows"]), int(g["cols"])))
    assert np.array_equal(dequant_nf4(st).view(np.uint16), g["out"].view(np.uint16))


def test_nf4_levels_are_the_references():
    # solution/kernels.py:38-41
    assert NF4_LEVELS.dtype == np.float32 and NF4_LEVELS[0] == -1.0 and NF4_LEVELS[-1] == 1.0
    assert NF4_LEVELS[7] == 0.0 and np.all(np.diff(NF4_LEVELS) > 0)


def test_nf4_quantise_round_trip():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((128, 256)) * 0.02).astype(np.float32)
    for nested in (False, True):
        st = quantize_nf4(w, nested=nested)
        back = dequant_nf4(st).astype(np.float32)
        # nearest level: error at most half the widest level gap (-1 .. -0.696) times the absmax
        err = np.abs(back - w).reshape(-1, 64).max(1)
        amax = np.abs(w).reshape(-1, 64).max(1)
        assert np.all(err <= 0.5 * 0.31 * amax * (1.05 if nested else 1.0) + 1e-6)


def test_philox_known_answer():
    # Random123 known-answer vectors for Philox4x32-10 (counter, key -> output)
    out = philox4x32_10(np.uint32([0]), np.uint32([0]), np.uint32([0]), np.uint32([0]),
                        np.uint32([0]), np.uint32([0]))
    assert [int(o[0]) for o in out] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    ff = np.uint32([0xFFFFFFFF])
    out = philox4x32_10(ff, ff, ff, ff, ff, ff)
    assert [int(o[0]) for o in out] == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]


def test_dropout_mask_bit_exact_vs_reference(golden):
    g = golden("dropout.npz")
    i = 0
    while f"case{i}" in g:
        seed, ctr, G, vec, n = (int(x) for x in g[f"case{i}"])
        keep = dropout_keep(np.arange(n), seed, ctr, G, float(g[f"p{i}"]), vec)
        assert np.array_equal(keep.astype(np.int8), g[f"keep{i}"]), i
        i += 1
    assert i >= 4


def test_dropout_draw_arithmetic():
    # solution/engine.py:787-797 on a 148-SM B200 (1184 resident 256-thread blocks)
    seed, ctr, thr, off = draw(4 * 512 * 1536, 0, 7, 1184)
    assert (ctr, thr, off) == (0, 1184 * 256, 12)
    seed, ctr, thr, off = draw(3 * 5 * 64, 16, 2**64 - 1, 1184)
    assert (seed, ctr, thr, off) == (-1, 4, 4 * 256, 20)  # ceil(960 / 256) = 4 blocks


def test_rms_vs_reference(golden):
    g = golden("rms.npz")
    kw = dict(tok=g["tok"], p=float(g["p"]), seed=int(g["seed"]), ctr_q=int(g["ctr_q"]),
              ctr_v=int(g["ctr_v"]), G=int(g["G"]))
    out = OK.rms_fwd(g["x"], g["w"], float(g["eps"]), delta=g["delta"].astype(np.float32), **kw)
    np.testing.assert_allclose(out["xsum"], g["xsum"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(out["rstd"], g["rstd"], rtol=1e-5)
    np.testing.assert_allclose(out["y"], g["y"].astype(np.float32), rtol=2e-3, atol=2e-3)
    assert np.array_equal(out["yq"] != 0, g["yq"] != 0)
    assert np.array_equal(out["yv"] != 0, g["yv"] != 0)
    dx = OK.rms_bwd(g["dy"], out["xsum"], out["rstd"], g["w"], dres=g["dres"], tq=g["tq"],
                    tv=g["tv"], grad_scale=float(g["grad_scale"]), **kw)
    np.testing.assert_allclose(dx, g["dx"], rtol=1e-4, atol=1e-4)


def test_rope_vs_reference(golden):
    g = golden("rope.npz")
    HQ, HKV, D = 12, 2, 128
    q, k, v = OK.rope_fwd(g["qkv"], g["cos"], g["sin"], g["pos"], HQ, HKV, D, float(g["scale"]),
                          lq=g["lq"], lv=g["lv"])
    np.testing.assert_allclose(q, g["q"].astype(np.float32), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(k, g["k"][:, ::HQ // HKV].astype(np.float32), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(v, g["v"][:, ::HQ // HKV].astype(np.float32), rtol=2e-3, atol=2e-3)
    dqkv = OK.rope_bwd(g["dq"], g["dk"], g["dv"], g["cos"], g["sin"], g["pos"], HQ, HKV, D)
    np.testing.assert_allclose(dqkv, g["dqkv"].astype(np.float32), rtol=1e-2, atol=1e-2)


def test_glu_vs_reference(golden):
    g = golden("glu.npz")
    np.testing.assert_allclose(OK.glu_fwd(g["gu"]), g["m"].astype(np.float32), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(OK.glu_bwd(g["dm"], g["gu"]), g["dgu"].astype(np.float32),
                               rtol=1e-2, atol=1e-2)


def test_ce_vs_reference(golden):
    g = golden("ce.npz")
    loss, ent, cor, grad = OK.ce_rows(g["logits"].astype(np.float32), g["target"])
    np.testing.assert_allclose(loss, g["loss"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(ent, g["entropy"], rtol=1e-3, atol=1e-3)
    assert np.array_equal(cor, g["correct"])
    np.testing.assert_allclose(grad, g["grad"].astype(np.float32), rtol=1e-3, atol=1e-3)


def test_integer_keep_threshold_equals_the_fp32_keep_test():
    """The kernels keep a Philox draw u iff u < ql_dropout_keep_threshold(p): the same set as the
    fp32 test u * 2^-32 + 2^-33 < p (solution/kernels.py:108-126), checked at the threshold and
    around it, and on a random sample of draws, for the dropout rates in use."""
    from hack_fe30cb28_opus_5_5_ultracode_b200 import _lib

    lib = _lib.lib()

    def keep(u, p):
        f = u.astype(np.float32) * np.float32(2.3283064365386963e-10) + np.float32(1.1641532182693481e-10)
        return f.astype(np.float32) < np.float32(p)

    rng = np.random.default_rng(5)
    for p_drop in (0.05, 0.1, 0.25, 0.3, 0.5, 0.9, 1e-7):
        p = np.float32(1.0 - p_drop)
        t = int(lib.ql_dropout_keep_threshold(float(p)))
        near = np.arange(max(t - 300, 0), min(t + 300, 2**32), dtype=np.uint64).astype(np.uint32)
        sample = rng.integers(0, 2**32, 100000, dtype=np.uint64).astype(np.uint32)
        for u in (near, sample):
            assert np.array_equal(keep(u, p), u < t), p_drop
    assert lib.ql_dropout_keep_threshold(1.0) == 0xFFFFFFFF

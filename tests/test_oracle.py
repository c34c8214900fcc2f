"""Pins the oracle (oracle/liboracle.so) before anything is checked against it.

1. Known-answer tests restated from the reference's own unit tests
   (engine/tests/ops_test.c, engine/tests/kv_cache_test.c).
2. Golden vectors produced by the reference implementation itself
   (tests/golden/make_golden.py): the oracle must be BIT-exact.
3. Where the reference build is present (oracle/_ref), fresh seeded random
   cross-checks, bit-exact.
"""
import math

import numpy as np
import pytest

from conftest import golden
from shukuchi_b200 import synth


def f16(x: float) -> int:
    return int(np.array([x], np.float16).view(np.uint16)[0])


# ---------------------------------------------------------------- KATs
def test_kat_q4k_single_block(oracle):
    # engine/tests/ops_test.c:86-117: d=1, dmin=0, sc=1, qs[0]=0xF0, x[0]=x[32]=1 -> 15
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.array([f16(1.0)], np.uint16).view(np.uint8)
    blk[2:4] = np.array([f16(0.0)], np.uint16).view(np.uint8)
    blk[4:16] = [1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1]
    blk[16] = 0xF0
    x = np.zeros(256, np.float32)
    x[0] = x[32] = 1.0
    y = oracle.matvec(12, blk, x, 1, 256)
    assert abs(y[0] - 15.0) <= 1e-3


def test_kat_rmsnorm(oracle):
    # engine/tests/ops_test.c:48-59
    x = np.array([1, 2, 3, 4], np.float32)
    y = oracle.rmsnorm(x, np.ones(4, np.float32))
    inv = 1.0 / math.sqrt((1 + 4 + 9 + 16) / 4 + 1e-5)
    np.testing.assert_allclose(y, x * inv, atol=1e-5)


def test_kat_rope(oracle):
    # engine/tests/ops_test.c:61-68: head_dim 2, pos 1 -> (cos 1, sin 1)
    y = oracle.rope(np.array([1.0, 0.0], np.float32), 1, 2, 1, 10000.0)
    assert abs(y[0] - math.cos(1.0)) <= 1e-5 and abs(y[1] - math.sin(1.0)) <= 1e-5


def test_kat_attention(oracle):
    # engine/tests/ops_test.c:119-141
    q = np.array([1, 0], np.float32)
    k = np.array([1, 0, 0, 1], np.float32)
    v = np.array([1, 2, 3, 4], np.float32)
    scale = 1.0 / math.sqrt(2.0)
    out = oracle.attention(q, k, v, 1, 1, 2, 2, np.float32(scale))
    s0, s1 = math.exp(scale), 1.0
    w0, w1 = s0 / (s0 + s1), s1 / (s0 + s1)
    np.testing.assert_allclose(out, [w0 * 1 + w1 * 3, w0 * 2 + w1 * 4], atol=1e-5)


def test_kat_swiglu_zero_weights(oracle):
    # engine/tests/ops_test.c:143-172: all-zero Q4_K gate/up/down -> 0
    w = np.zeros(256 * 144, np.uint8)
    x = (np.arange(256, dtype=np.float32) * 0.01)
    g = oracle.matvec(12, w, x, 256, 256)
    u = oracle.matvec(12, w, x, 256, 256)
    y = oracle.matvec(12, w, oracle.swiglu(g, u), 256, 256)
    assert np.all(np.abs(y) <= 1e-6)


def test_kat_kv_roundtrip(oracle):
    # engine/tests/kv_cache_test.c:15-53: 2 KV heads x hd 4, block 4, 4 tokens, tol 0.05
    kv = oracle.kv_create(1, 2, 4, 8, block=4)
    try:
        import ctypes as C
        for t in range(4):
            k = np.array([(t * 10 + i) * 0.1 for i in range(8)], np.float32)
            v = -k
            assert oracle.L.orc_kv_append(kv, 0, t, k.ctypes.data, v.ctypes.data) == 0
        ko = np.zeros(32, np.float32)
        vo = np.zeros(32, np.float32)
        assert oracle.L.orc_kv_read_range(kv, 0, 0, 4, ko.ctypes.data, vo.ctypes.data) == 0
        exp = np.array([(t * 10 + i) * 0.1 for t in range(4) for i in range(8)], np.float32)
        assert np.all(np.abs(ko - exp) <= 0.05) and np.all(np.abs(vo + exp) <= 0.05)
        assert oracle.L.orc_kv_seq_len(kv, 0) == 4
        oracle.L.orc_kv_clear(kv)
        assert oracle.L.orc_kv_seq_len(kv, 0) == 0
    finally:
        oracle.kv_destroy(kv)


def test_half_subnormal_quirk(oracle):
    # engine/src/ops.c:65-78 decodes fp16 subnormals at half the IEEE value
    for h in (0x0001, 0x0155, 0x03FF, 0x8001):
        ieee = float(np.array([h], np.uint16).view(np.float16)[0])
        assert oracle.half_to_float(h) == ieee / 2
    for h in (0x0400, 0x3C00, 0x7BFF, 0x0000):
        assert oracle.half_to_float(h) == float(np.array([h], np.uint16).view(np.float16)[0])


# ------------------------------------------------------------- goldens
def test_golden_gemv(oracle):
    for name, qt in (("gemv_q4k", 12), ("gemv_q5k", 13), ("gemv_q6k", 14)):
        g = golden(name)
        y = oracle.matvec(qt, g["w"], g["x"], int(g["m"]), int(g["k"]))
        assert np.array_equal(y.view(np.uint32), g["y"].view(np.uint32)), name


def test_golden_q8(oracle):
    g = golden("q8")
    assert np.array_equal(oracle.q8_quantize(g["x"]), g["blocks"])


def test_golden_rmsnorm_rope(oracle):
    g = golden("rmsnorm")
    assert np.array_equal(oracle.rmsnorm(g["x"], g["w"]), g["y"])
    g = golden("rope")
    y = oracle.rope(g["x"], int(g["n_heads"]), int(g["head_dim"]), int(g["pos"]))
    assert np.array_equal(y, g["y"])


def test_golden_attention(oracle):
    g = golden("attention")
    H, KV, hd, seq = (int(v) for v in g["dims"])
    out = oracle.attention(g["q"], g["k"], g["v"], H, KV, hd, seq, np.float32(1.0 / np.sqrt(hd)))
    assert np.array_equal(out, g["out"])


def test_golden_embed(oracle):
    g = golden("embed")
    assert np.array_equal(oracle.embed(g["table"], 12, int(g["token"]), 512), g["out"])


def test_golden_tiny_model(oracle):
    g = golden("tiny_model")
    model = synth.make_model("tiny", seed=int(g["seed"]))
    assert model.digest().encode() == g["digest"].tobytes(), "synthetic weight stream changed"
    toks, logits = oracle.generate(model, g["prompt"], len(g["tokens"]))
    assert np.array_equal(toks, g["tokens"])
    assert np.array_equal(logits, g["logits"])


# ------------------------------------------- live cross-check vs the reference
@pytest.mark.parametrize("qt,m,k", [(12, 33, 768), (14, 33, 768), (14, 5, 5632), (12, 3, 2048), (13, 33, 768), (13, 4, 5632)])
def test_live_gemv_vs_reference(oracle, reference, qt, m, k):
    rng = np.random.default_rng(m * 7 + k)
    w = synth.quant_matrix(rng, qt, m, k)
    x = rng.normal(0, 2, k).astype(np.float32)
    a = oracle.matvec(qt, w, x, m, k)
    b = reference.matvec(qt, w, x, m, k)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_live_ops_vs_reference(oracle, reference):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, 1024).astype(np.float32)
    assert np.array_equal(oracle.q8_quantize(x), reference.q8_quantize(x))
    w = (1 + rng.normal(0, 0.02, 1024)).astype(np.float32)
    assert np.array_equal(oracle.rmsnorm(x, w), reference.rmsnorm(x, w))
    for pos in (0, 1, 2047, 40000):
        assert np.array_equal(oracle.rope(x, 8, 128, pos), reference.rope(x, 8, 128, pos))


def test_live_model_vs_reference(oracle, reference):
    import importlib.util, os
    spec = importlib.util.spec_from_file_location(
        "mg", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    model = synth.make_model("small", seed=11)
    prompt = np.array([5, 17, 1000, 3], np.uint32)
    t_ref, l_ref = mg.tiny_generate(reference, model, prompt, 5)
    t_orc, l_orc = oracle.generate(model, prompt, 5)
    assert np.array_equal(t_ref, t_orc)
    assert np.array_equal(l_ref, l_orc)


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_conditioned_weights_are_unit_gain(oracle, qt):
    """synth's conditioned matrices (used by the multi-position layer and
    prefill tests): dequantised by the oracle they are zero-mean with rms
    about 1/sqrt(cols), so a matvec keeps activations of order one; the
    Q4_K / Q5_K blocks carry mins equal to their scales.  (Blocks whose fp16
    d is subnormal decode d at half its value -- the reference's quirk -- while
    dmin = 7.5 d or 15.5 d is normal, so those blocks are not centred: a small
    mean remains, largest for Q5_K, whose d are smallest.)"""
    rng = np.random.default_rng(qt)
    rows, cols = 64, 1024
    w = synth.quant_matrix(rng, qt, rows, cols, conditioned=True)
    d = oracle.dequant(qt, w, rows * cols).astype(np.float64)
    target = 1.0 / math.sqrt(cols)
    assert abs(d.mean()) < 0.25 * target
    assert 0.8 * target < d.std() < 1.25 * target
    if qt in (12, 13):
        b = w.reshape(-1, synth.BLOCK_BYTES[qt])
        sc = b[:, 4:16]
        assert np.array_equal(sc[:, 4:8], sc[:, 0:4])
        assert np.array_equal(sc[:, 8:12] >> 4, sc[:, 8:12] & 0xF)

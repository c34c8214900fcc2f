"""Glue ops on the GPU vs the oracle: embedding (bit-exact, same per-element
expression), argmax (first index on ties), RMSNorm / RoPE / SwiGLU (fp32
tolerance; CUDA's sinf/cosf/powf/expf differ from glibc by a few ulp)."""
import numpy as np
import pytest
import torch

from conftest import golden, to_dev
from shukuchi_b200 import synth

pytestmark = pytest.mark.gpu


def test_embed_bit_exact(oracle, ctx):
    g = golden("embed")
    out = torch.zeros(512, device="cuda")
    table_d = to_dev(g["table"])  # keep the device copy alive until the kernel ran
    ctx.embed(table_d.data_ptr(), 12, 10, int(g["token"]), out.data_ptr(), 512)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), g["out"])
    rng = np.random.default_rng(1)
    table = synth.quant_matrix(rng, 12, 50, 2048)
    td = to_dev(table)
    for tok in (0, 17, 49):
        o = torch.zeros(2048, device="cuda")
        ctx.embed(td.data_ptr(), 12, 50, tok, o.data_ptr(), 2048)
        torch.cuda.synchronize()
        assert np.array_equal(o.cpu().numpy(), oracle.embed(table, 12, tok, 2048))


def test_embed_rejects_bad_token(ctx):
    from shukuchi_b200.cuda import ShkError
    t = torch.zeros(144 * 4, dtype=torch.uint8, device="cuda")
    o = torch.zeros(256, device="cuda")
    with pytest.raises(ShkError):
        ctx.embed(t.data_ptr(), 12, 4, 4, o.data_ptr(), 256)


@pytest.mark.parametrize("n", [1, 7, 32000, 128256])
def test_argmax_first_index(oracle, ctx, n):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 1, n).astype(np.float32)
    if n > 10:
        m = x.max() + 1.0
        x[n // 3] = m
        x[n // 2] = m  # tie: the earlier index wins
        x[n - 1] = m
    xd = to_dev(x)
    assert ctx.argmax(xd.data_ptr(), n) == oracle.argmax(x)


@pytest.mark.parametrize("case", ["nan_first", "nan_block_start", "all_nan", "nan_then_max"])
def test_argmax_nan_like_the_reference(oracle, ctx, case):
    # engine/src/engine.c:424-431 keeps best = 0 while x[best] is NaN (nothing
    # compares greater) and skips NaN elements once best is a number
    n = 3 * 4096 + 77
    x = np.random.default_rng(5).normal(0, 1, n).astype(np.float32)
    if case == "nan_first":
        x[0] = np.nan
        x[5000] = 50.0
    elif case == "nan_block_start":
        x[4096] = np.nan
        x[4097] = 40.0
    elif case == "all_nan":
        x[:] = np.nan
    else:
        x[100:200] = np.nan
        x[8000] = 60.0
    xd = to_dev(x)
    assert ctx.argmax(xd.data_ptr(), n) == oracle.argmax(x)


def test_rmsnorm(oracle, ctx):
    rng = np.random.default_rng(2)
    for d in (256, 2048, 4096, 8192):
        x = rng.normal(0, 5, d).astype(np.float32)
        w = (1 + rng.normal(0, 0.02, d)).astype(np.float32)
        y = torch.zeros(d, device="cuda")
        xd, wd = to_dev(x), to_dev(w)
        ctx.rmsnorm(xd.data_ptr(), wd.data_ptr(), y.data_ptr(), d)
        torch.cuda.synchronize()
        # sum of squares in a different order: 1/sqrt(mean) agrees to ~sqrt(d)*eps
        np.testing.assert_allclose(y.cpu().numpy(), oracle.rmsnorm(x, w), rtol=3e-5, atol=1e-7)


@pytest.mark.parametrize("pos", [0, 1, 37, 2047, 32767])
def test_rope(oracle, ctx, pos):
    rng = np.random.default_rng(pos)
    for nh, hd in ((4, 64), (8, 128)):
        x = rng.normal(0, 1, nh * hd).astype(np.float32)
        xd = to_dev(x)
        ctx.rope(xd.data_ptr(), nh, hd, pos, 10000.0)
        torch.cuda.synchronize()
        np.testing.assert_allclose(xd.cpu().numpy(), oracle.rope(x, nh, hd, pos), rtol=0, atol=2e-5)


def test_swiglu(oracle, ctx):
    rng = np.random.default_rng(4)
    g = rng.normal(0, 4, 5000).astype(np.float32)
    u = rng.normal(0, 4, 5000).astype(np.float32)
    h = torch.zeros(5000, device="cuda")
    gd, ud = to_dev(g), to_dev(u)
    ctx.swiglu(gd.data_ptr(), ud.data_ptr(), h.data_ptr(), 5000)
    torch.cuda.synchronize()
    np.testing.assert_allclose(h.cpu().numpy(), oracle.swiglu(g, u), rtol=2e-6, atol=1e-6)


def test_bounded_wait_times_out_and_context_survives(oracle, ctx):
    """A device wait that nothing satisfies ends after its budget with
    SHK_ETIMEOUT (no hang, no trap); the same context then runs a GEMV."""
    import time

    from shukuchi_b200 import cuda as sc
    t0 = time.monotonic()
    rc = sc.lib().shk_cuda_selftest_wait_timeout(ctx.h, 20000)  # 20 ms
    assert time.monotonic() - t0 < 10.0
    assert rc == -5  # SHK_ETIMEOUT
    ctx.check()  # error word was cleared by the report
    rng = np.random.default_rng(2)
    w = synth.quant_matrix(rng, 12, 64, 512)
    x = rng.standard_normal(512).astype(np.float32)
    y = torch.zeros(64, device="cuda")
    wd, xd = to_dev(w), to_dev(x)
    ctx.matmul(12, wd.data_ptr(), xd.data_ptr(), y.data_ptr(), 64, 512)
    torch.cuda.synchronize()
    ref = oracle.matvec(12, w, x, 64, 512)
    assert np.allclose(y.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)

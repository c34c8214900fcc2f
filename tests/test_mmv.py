"""Tensor-core matvec over row-tiled weights (SHK_DTYPE_Q4_K_TILED /
SHK_DTYPE_Q6_K_TILED) against the oracle's op_matmul_q4_k / op_matmul_q6_k,
and the tiled layout byte for byte against a numpy restatement.

Tolerance: per row |dy| <= 4*sqrt(k)*2^-24 * sum|w*x| (two fp32 summation
orders), the same bound as the staged GEMV's tests."""
import numpy as np
import pytest
import torch

from conftest import gemv_tolerance, to_dev
from shukuchi_b200 import synth

BB = {12: 144, 14: 210}
TB = {12: 16 * 144, 14: 16 * 210}


def tile_ref(w: np.ndarray, qt: int, m: int, k: int) -> np.ndarray:
    """The row-tiled layout, restated in numpy (include/shk_cuda.h): tiles of
    16 rows x one super-block, [row tile][block], rows past m zero."""
    nb = k // 256
    nt = (m + 15) // 16
    rows = np.zeros((nt * 16, nb, BB[qt]), np.uint8)
    rows[:m] = np.asarray(w, np.uint8).reshape(m, nb, BB[qt])
    R = rows.reshape(nt, 16, nb, BB[qt])
    if qt == 12:
        hdr = R[..., :16].transpose(0, 2, 1, 3)                       # t, b, row, 16
        qs = R[..., 16:].reshape(nt, 2, 8, nb, 4, 4, 8)              # t, h, g, b, j, t4, e
        qs = qs.transpose(0, 3, 4, 2, 5, 1, 6)                       # t, b, j, g, t4, h, e
        out = np.concatenate([hdr.reshape(nt, nb, -1), qs.reshape(nt, nb, -1)], axis=2)
    else:
        ql = R[..., :128].reshape(nt, 2, 8, nb, 2, 2, 4, 8)          # t, h, g, b, n, c, t4, e
        ql = ql.transpose(0, 3, 4, 2, 6, 1, 5, 7).reshape(nt, nb, 2, 8, 4, 2, 16)
        qh = R[..., 128:192].reshape(nt, 2, 8, nb, 2, 4, 8)          # t, h, g, b, n, t4, e
        qh = qh.transpose(0, 3, 4, 2, 5, 1, 6)                       # t, b, n, g, t4, h, e
        quants = np.concatenate([ql, qh], axis=6)                    # t, b, n, g, t4, h, 24
        sc = R[..., 192:208].transpose(0, 2, 1, 3)
        d = R[..., 208:210].transpose(0, 2, 1, 3)
        out = np.concatenate([quants.reshape(nt, nb, -1), sc.reshape(nt, nb, -1), d.reshape(nt, nb, -1)], axis=2)
    assert out.shape[2] == TB[qt]
    return out.reshape(-1)


def test_tile_ref_is_a_permutation():
    """CPU check of the restatement itself: every byte of a full tile comes
    from exactly one source byte."""
    for qt in (12, 14):
        m, k = 32, 512
        n = m * (k // 256) * BB[qt]
        src = np.arange(n, dtype=np.int64)
        # permutation of indices: tile the index array bytewise via 3 base-256 digits
        digits = [(src >> (8 * i)) & 0xFF for i in range(3)]
        tiled = [tile_ref(d.astype(np.uint8), qt, m, k).astype(np.int64) for d in digits]
        back = tiled[0] | (tiled[1] << 8) | (tiled[2] << 16)
        assert np.array_equal(np.sort(back), src)


def _tile_dev(ctx, qt, w, m, k):
    from shukuchi_b200 import cuda as sc
    src = to_dev(w)
    dst = torch.empty(sc.tiled_bytes(qt, m, k), dtype=torch.uint8, device="cuda")
    ctx.tile(qt, src.data_ptr(), m, k, dst.data_ptr())
    ctx.sync()
    return dst


def _check(oracle, ctx, qt, m, k, seed, xscale=1.0, x=None, subnormal=False):
    from shukuchi_b200 import cuda as sc
    rng = np.random.default_rng(seed)
    blocks = (synth.q4k_blocks if qt == 12 else synth.q6k_blocks)(rng, m * (k // 256))
    if subnormal:
        from golden.make_golden import subnormal_scales
        subnormal_scales(blocks, qt, rng, frac=0.7)
    w = blocks.reshape(-1)
    if x is None:
        x = (rng.normal(0, 1, k) * xscale).astype(np.float32)
    t = _tile_dev(ctx, qt, w, m, k)
    assert np.array_equal(t.cpu().numpy(), tile_ref(w, qt, m, k)), "tiled bytes differ"
    xd = to_dev(x)
    y = torch.full((m,), float("nan"), device="cuda")
    dt = sc.DTYPE_Q4_K_TILED if qt == 12 else sc.DTYPE_Q6_K_TILED
    ctx.matvec(dt, t.data_ptr(), xd.data_ptr(), y.data_ptr(), m, k)
    ctx.sync()
    ctx.check()
    yr = oracle.matvec(qt, w, x, m, k)
    tol = gemv_tolerance(oracle, qt, w, x, m, k)
    err = np.abs(y.cpu().numpy().astype(np.float64) - yr)
    assert np.all(err <= tol), (float(np.max(err / tol)), int(np.argmax(err / tol)))


@pytest.mark.gpu
@pytest.mark.parametrize("m,k", [(1, 256), (16, 256), (7, 512), (64, 2048), (333, 1024), (1024, 4096),
                                 (4096, 4096), (1000, 14336), (3, 8192), (4096, 14336), (14336, 4096),
                                 (37, 28672), (9475, 4096), (2048, 5632)])
def test_q4k_tiled(oracle, ctx, m, k):
    _check(oracle, ctx, 12, m, k, seed=m + k)


@pytest.mark.gpu
@pytest.mark.parametrize("m,k", [(1, 256), (9, 512), (256, 2048), (1024, 4096), (777, 4096),
                                 (4096, 14336), (100, 5632), (64, 1792), (5, 3584), (37, 28672),
                                 (2000, 4096)])
def test_q6k_tiled(oracle, ctx, m, k):
    _check(oracle, ctx, 14, m, k, seed=m * 3 + k)


@pytest.mark.gpu
@pytest.mark.parametrize("qt", [12, 14])
def test_tiled_subnormal_scales(oracle, ctx, qt):
    _check(oracle, ctx, qt, 64, 1024, seed=99, subnormal=True)


@pytest.mark.gpu
@pytest.mark.parametrize("qt", [12, 14])
def test_tiled_large_and_tiny_inputs(oracle, ctx, qt):
    _check(oracle, ctx, qt, 128, 2048, seed=5, xscale=1e6)
    _check(oracle, ctx, qt, 128, 2048, seed=6, xscale=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("qt", [12, 14])
def test_tiled_outlier_in_block(oracle, ctx, qt):
    """x is fixed point relative to each 256-element block's maximum: a block
    whose maximum is a 1000x outlier keeps the small elements' error inside the
    per-row bound (which grows with sum |w x|, outlier included)."""
    rng = np.random.default_rng(11)
    k = 4096
    x = rng.normal(0, 1, k).astype(np.float32)
    for b in (0, 5, 15):
        x[256 * b + 17] = 1000.0 * (1 if b % 2 else -1)
    _check(oracle, ctx, qt, 300, k, seed=12, x=x)


@pytest.mark.gpu
def test_tile_rejects_bad_arguments(ctx):
    from shukuchi_b200.cuda import ShkError
    d = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(ShkError):
        ctx.tile(12, d.data_ptr(), 1, 100, d.data_ptr())  # k % 256
    with pytest.raises(ShkError):
        ctx.tile(13, d.data_ptr(), 1, 256, d.data_ptr())  # not Q4_K / Q6_K

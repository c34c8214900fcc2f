"""Q4_K / Q5_K / Q6_K dequantise-matvec on the GPU vs the oracle (op_matmul_q4_k
/ op_matmul_q5_k / op_matmul_q6_k restated).  Tolerance: per row |dy| <= 4*sqrt(k)*2^-24 * sum|w*x|
(two fp32 summation orders)."""
import numpy as np
import pytest
import torch

from conftest import gemv_tolerance, golden, to_dev
from shukuchi_b200 import synth

pytestmark = pytest.mark.gpu


def run_gemv(ctx, qt, w, x, m, k):
    wd, xd = to_dev(w), to_dev(x)
    yd = torch.full((m,), float("nan"), device="cuda")
    ctx.matmul(qt, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), m, k,
               stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.check()
    return yd.cpu().numpy()


def check(oracle, ctx, qt, m, k, seed, subnormal=False, xscale=1.0):
    rng = np.random.default_rng(seed)
    blocks = {12: synth.q4k_blocks, 13: synth.q5k_blocks, 14: synth.q6k_blocks}[qt](rng, m * (k // 256))
    if subnormal:
        from golden.make_golden import subnormal_scales
        subnormal_scales(blocks, qt, rng, frac=0.7)
    w = blocks.reshape(-1)
    x = (rng.normal(0, 1, k) * xscale).astype(np.float32)
    y = run_gemv(ctx, qt, w, x, m, k)
    yr = oracle.matvec(qt, w, x, m, k)
    tol = gemv_tolerance(oracle, qt, w, x, m, k)
    err = np.abs(y.astype(np.float64) - yr)
    assert np.all(err <= tol), (np.max(err / tol), int(np.argmax(err / tol)))


@pytest.mark.parametrize("m,k", [(1, 256), (7, 512), (64, 2048), (333, 1024), (1024, 4096),
                                 (4096, 4096), (1000, 14336), (3, 8192), (4096, 14336), (14336, 4096),
                                 (37, 28672), (5, 65536), (9475, 4096)])
def test_q4k(oracle, ctx, m, k):
    # k > 8192 (more than 32 blocks a row): rows are split over warps in K slices
    check(oracle, ctx, 12, m, k, seed=m + k)


@pytest.mark.parametrize("m,k", [(1, 256), (9, 512), (256, 2048), (1024, 4096), (777, 4096),
                                 (4096, 14336), (100, 5632), (64, 1792), (5, 3584), (37, 28672), (3, 65536)])
def test_q6k(oracle, ctx, m, k):
    # 5632 / 1792 / 3584 give rows that are not 16-byte multiples: plain-load kernel
    check(oracle, ctx, 14, m, k, seed=m * 3 + k)


@pytest.mark.parametrize("m,k", [(1, 256), (2, 512), (3, 1280), (64, 2048), (333, 1024), (4096, 4096),
                                 (1000, 14336), (4096, 14336), (37, 28672), (5, 64512)])
def test_q5k(oracle, ctx, m, k):
    # the reference's own Q5_K element order (engine/src/ops.c:144-165); odd m
    # (a last row pair of one row), 5 blocks a row (a partial 4-block step),
    # k up to the largest x the kernel holds in shared memory
    check(oracle, ctx, 13, m, k, seed=m * 5 + k)


def test_q5k_rejects_too_long_rows(ctx):
    from shukuchi_b200.cuda import ShkError
    d = torch.zeros(65536 * 176 // 256, dtype=torch.uint8, device="cuda")
    x = torch.zeros(65536, device="cuda")
    with pytest.raises(ShkError):
        ctx.matmul(13, d.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 65536)


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_subnormal_scales(oracle, ctx, qt):
    # the reference decodes subnormal fp16 scales at half value; GPU must too
    check(oracle, ctx, qt, 64, 1024, seed=99, subnormal=True)


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_large_and_tiny_inputs(oracle, ctx, qt):
    check(oracle, ctx, qt, 128, 2048, seed=5, xscale=1e6)
    check(oracle, ctx, qt, 128, 2048, seed=6, xscale=1e-6)


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_outlier_in_block(oracle, ctx, qt):
    # x is fixed point relative to each 256-element block's maximum; a 1000x
    # outlier in a block must keep the row inside the per-row bound
    rng = np.random.default_rng(11)
    m, k = 300, 4096
    w = synth.quant_matrix(rng, qt, m, k)
    x = rng.normal(0, 1, k).astype(np.float32)
    for b in (0, 5, 15):
        x[256 * b + 17] = 1000.0 * (1 if b % 2 else -1)
    y = run_gemv(ctx, qt, w, x, m, k)
    tol = gemv_tolerance(oracle, qt, w, x, m, k)
    assert np.all(np.abs(y.astype(np.float64) - oracle.matvec(qt, w, x, m, k)) <= tol)


def test_golden_vectors(oracle, ctx):
    for name, qt in (("gemv_q4k", 12), ("gemv_q5k", 13), ("gemv_q6k", 14)):
        g = golden(name)
        m, k = int(g["m"]), int(g["k"])
        y = run_gemv(ctx, qt, g["w"], g["x"], m, k)
        tol = gemv_tolerance(oracle, qt, g["w"], g["x"], m, k)
        assert np.all(np.abs(y.astype(np.float64) - g["y"]) <= tol), name


def test_host_pointer_variant(oracle, ctx):
    rng = np.random.default_rng(3)
    for qt in (12, 13, 14):
        m, k = 300, 4096
        w = synth.quant_matrix(rng, qt, m, k)
        x = rng.normal(0, 1, k).astype(np.float32)
        y = np.zeros(m, np.float32)
        ctx.matmul_host(qt, w, x, y, m, k)
        tol = gemv_tolerance(oracle, qt, w, x, m, k)
        assert np.all(np.abs(y.astype(np.float64) - oracle.matvec(qt, w, x, m, k)) <= tol)


def test_rejects_bad_shapes(ctx):
    from shukuchi_b200.cuda import ShkError
    d = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(ShkError):
        ctx.matmul(12, d.data_ptr(), d.data_ptr(), d.data_ptr(), 1, 100)  # k % 256


def planar_ref(rows: np.ndarray, nb: int, stride: int) -> np.ndarray:
    """The planar Q6_K row layout, restated in numpy: rows (GGUF blocks,
    `stride` bytes apart) regrouped as [ql][qh][scales][d] with the 16-byte
    chunks of block b rotated (ql chunk c at slot (c + b) & 7, qh chunk c at
    slot (c + (b >> 1)) & 3)."""
    out = rows.copy()
    for r in range(rows.shape[0]):
        src = rows[r]
        dst = out[r]
        for b in range(nb):
            blk = src[210 * b:210 * b + 210]
            for c in range(8):
                s = ((c + b) & 7) * 16
                dst[128 * b + s:128 * b + s + 16] = blk[16 * c:16 * c + 16]
            for c in range(4):
                s = ((c + (b >> 1)) & 3) * 16
                dst[128 * nb + 64 * b + s:128 * nb + 64 * b + s + 16] = blk[128 + 16 * c:128 + 16 * c + 16]
            dst[192 * nb + 16 * b:192 * nb + 16 * b + 16] = blk[192:208]
            dst[208 * nb + 2 * b:208 * nb + 2 * b + 2] = blk[208:210]
    return out


@pytest.mark.parametrize("m,k", [(3, 256), (17, 4096), (5, 5632), (2, 14336)])
def test_q6k_planar_layout_and_matvec(oracle, ctx, m, k):
    """shk_cuda_q6k_repack writes exactly the planar layout (byte for byte),
    the inverse restores the GGUF blocks, and the staged GEMV on planar rows
    (padded strides included) matches the oracle on the GGUF bytes."""
    from shukuchi_b200 import cuda as sc
    rng = np.random.default_rng(m + k)
    nb = k // 256
    w = synth.quant_matrix(rng, 14, m, k).reshape(m, 210 * nb)
    stride = (210 * nb + 15) // 16 * 16
    rows = np.zeros((m, stride), np.uint8)
    rows[:, :210 * nb] = w
    d = to_dev(rows.reshape(-1))
    ctx.q6k_repack(d.data_ptr(), m, k, stride, True)
    ctx.sync()
    assert np.array_equal(d.cpu().numpy().reshape(m, stride), planar_ref(rows, nb, stride))
    x = rng.normal(0, 1, k).astype(np.float32)
    xd = to_dev(x)
    y = torch.full((m,), float("nan"), device="cuda")
    ctx.matvec(sc.DTYPE_Q6_K_PLANAR, d.data_ptr(), xd.data_ptr(), y.data_ptr(), m, k, row_stride=stride)
    ctx.sync()
    ctx.check()
    wf = w.reshape(-1)
    tol = gemv_tolerance(oracle, 14, wf, x, m, k)
    assert np.all(np.abs(y.cpu().numpy().astype(np.float64) - oracle.matvec(14, wf, x, m, k)) <= tol)
    ctx.q6k_repack(d.data_ptr(), m, k, stride, False)
    ctx.sync()
    assert np.array_equal(d.cpu().numpy().reshape(m, stride), rows)

"""Batched prefill matmul on the tensor cores (tcgen05, f16 x f16 -> fp32)
vs an fp64 product of the oracle-dequantised weights.

The contraction is the one n_tokens calls of op_matmul_q4_k / op_matmul_q6_k
(engine/src/ops.c:266-314, 361-404) compute; the weights are rounded to f16
and each token's activations, scaled by a power of two, too (relative error
<= 2^-11 each; weights in the f16 subnormal range to within 2^-25), so each
output is bounded by 2^-9 * sum_k |w_k x_k| + 2^-24 * sum_k |x_k| (products
within 2^-10, fp32 accumulation)."""
import numpy as np
import pytest
import torch

from conftest import to_dev
from shukuchi_b200 import cuda as sc
from shukuchi_b200 import synth

pytestmark = pytest.mark.gpu


def _deq(oracle, qt, w, m, k):
    rb = (k // 256) * synth.BLOCK_BYTES[qt]
    return np.stack([oracle.dequant(qt, w[r * rb:(r + 1) * rb], k) for r in range(m)]).astype(np.float64)


@pytest.mark.parametrize("qt,m,k,t", [(12, 300, 1024, 200), (12, 128, 256, 1), (12, 77, 4096, 129),
                                      (14, 130, 2048, 64), (14, 64, 5632, 129), (14, 256, 4096, 256)])
def test_prefill_matches_dense_product(oracle, ctx, qt, m, k, t):
    rng = np.random.default_rng(m + k + t)
    w = synth.quant_matrix(rng, qt, m, k)
    x = rng.normal(0, 1, (t, k)).astype(np.float32)
    nb = k // 256
    rb = nb * synth.BLOCK_BYTES[qt]
    stride = (rb + 15) // 16 * 16
    rows = np.zeros((m, stride), np.uint8)
    rows[:, :rb] = w.reshape(m, rb)
    wd = to_dev(rows.reshape(-1))
    dt = qt
    if qt == 14:
        ctx.q6k_repack(wd.data_ptr(), m, k, stride, True)
        dt = sc.DTYPE_Q6_K_PLANAR
    xd = to_dev(x)
    y = torch.full((t, m), float("nan"), device="cuda")
    ctx.prefill_matmul(dt, wd.data_ptr(), xd.data_ptr(), y.data_ptr(), m, k, t, row_stride=stride)
    ctx.sync()
    ctx.check()
    W = _deq(oracle, qt, w, m, k)
    ref = x.astype(np.float64) @ W.T
    ax = np.abs(x).astype(np.float64)
    bound = (ax @ np.abs(W).T) * 2.0 ** -9 + ax.sum(axis=1, keepdims=True) * 2.0 ** -24 + 1e-6
    got = y.cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - ref) <= bound), float(np.max(np.abs(got - ref) / bound))


def test_prefill_token_rows_of_any_magnitude(oracle, ctx):
    """Token rows of magnitude 1e6 (beyond f16's 65504 unscaled), 1e-7 (f16
    subnormal unscaled), zero, and one with a single outlier: the per-token
    power-of-two scale keeps each row's relative bound."""
    m, k, t = 128, 1024, 5
    rng = np.random.default_rng(5)
    w = synth.quant_matrix(rng, 12, m, k)
    x = rng.normal(0, 1, (t, k)).astype(np.float32)
    x[0] *= 1e6
    x[1] *= 1e-7
    x[2] = 0.0
    x[3, 17] = 3e4
    wd = to_dev(w)
    xd = to_dev(x)
    y = torch.full((t, m), float("nan"), device="cuda")
    ctx.prefill_matmul(12, wd.data_ptr(), xd.data_ptr(), y.data_ptr(), m, k, t)
    ctx.sync()
    ctx.check()
    W = _deq(oracle, 12, w, m, k)
    ref = x.astype(np.float64) @ W.T
    ax = np.abs(x).astype(np.float64)
    bound = (ax @ np.abs(W).T) * 2.0 ** -9 + ax.sum(axis=1, keepdims=True) * 2.0 ** -24
    got = y.cpu().numpy().astype(np.float64)
    assert np.all(got[2] == 0.0)
    assert np.all(np.abs(got - ref) <= bound), float(np.max(np.abs(got - ref) / np.maximum(bound, 1e-300)))


def test_prefill_rejects_bad_arguments(ctx):
    from shukuchi_b200.cuda import ShkError
    d = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256, device="cuda")
    y = torch.zeros(4, device="cuda")
    with pytest.raises(ShkError):  # GGUF-layout Q6_K is not taken: repack first
        ctx.prefill_matmul(14, d.data_ptr(), x.data_ptr(), y.data_ptr(), 1, 256, 1)
    with pytest.raises(ShkError):  # k % 256
        ctx.prefill_matmul(12, d.data_ptr(), x.data_ptr(), y.data_ptr(), 1, 100, 1)

"""Q8_0 KV cache on the GPU: appended blocks must be BIT-identical to the
reference quantiser (q8_quantize_vec) for identical fp32 input; attention over
the cache vs the oracle (kv_cache_read_range + op_attention), relative
tolerance 2e-5 of max|out| per head."""
import numpy as np
import pytest
import torch

from conftest import to_dev
from shukuchi_b200 import cuda as sc

pytestmark = pytest.mark.gpu


def kv_inputs(rng, T, KV, hd):
    k = rng.normal(0, 1, (T, KV * hd)).astype(np.float32)
    v = rng.normal(0, 1, (T, KV * hd)).astype(np.float32)
    # exercise: an all-zero block (scale 1), exact .5 ties, a saturating value
    k[0, :32] = 0.0
    v[min(1, T - 1), 32:64] = (np.arange(32) - 16) * 0.5 + 0.25
    k[T - 1, 5] = 1e30
    return k, v


@pytest.mark.parametrize("KV,hd,start,T", [(8, 128, 0, 300), (4, 64, 17, 70000)])
def test_append_range_bit_exact(oracle, ctx, KV, hd, start, T):
    # bulk append (prefill-style) == per-position q8_quantize_vec; 70000
    # positions take two launches (grid.y <= 65535)
    rng = np.random.default_rng(T)
    k, v = kv_inputs(rng, T, KV, hd)
    kv = sc.KvCache(ctx, 1, KV, hd, start + T)
    try:
        kd, vd = to_dev(k), to_dev(v)
        kv.append_range(0, start, T, kd.data_ptr(), vd.data_ptr())
        nb = KV * hd // 32 * 36
        kb = torch.zeros(T * nb, dtype=torch.uint8, device="cuda")
        vb = torch.zeros_like(kb)
        kv.read_blocks(0, start, start + T, kb.data_ptr(), vb.data_ptr())
        torch.cuda.synchronize()
        ctx.check()
        ref_k = oracle.q8_quantize(k.reshape(-1))
        ref_v = oracle.q8_quantize(v.reshape(-1))
        assert np.array_equal(kb.cpu().numpy(), ref_k)
        assert np.array_equal(vb.cpu().numpy(), ref_v)
        assert kv.seq_len(0) == start + T
        with pytest.raises(sc.ShkError):
            kv.append_range(0, start + 1, T, kd.data_ptr(), vd.data_ptr())  # past max_seq
    finally:
        kv.close()


@pytest.mark.parametrize("KV,hd", [(2, 64), (8, 128), (4, 64)])
def test_append_bit_exact(oracle, ctx, KV, hd):
    rng = np.random.default_rng(KV * hd)
    T = 40
    k, v = kv_inputs(rng, T, KV, hd)
    kv = sc.KvCache(ctx, 2, KV, hd, 64)
    try:
        kd, vd = to_dev(k), to_dev(v)
        for t in range(T):
            kv.append(1, t, kd[t].data_ptr(), vd[t].data_ptr())
        nb = KV * hd // 32 * 36
        kb = torch.zeros(T * nb, dtype=torch.uint8, device="cuda")
        vb = torch.zeros_like(kb)
        kv.read_blocks(1, 0, T, kb.data_ptr(), vb.data_ptr())
        torch.cuda.synchronize()
        ctx.check()
        ref_k = np.concatenate([oracle.q8_quantize(k[t]) for t in range(T)])
        ref_v = np.concatenate([oracle.q8_quantize(v[t]) for t in range(T)])
        assert np.array_equal(kb.cpu().numpy(), ref_k)
        assert np.array_equal(vb.cpu().numpy(), ref_v)
        assert kv.seq_len(1) == T and kv.seq_len(0) == 0
        # read_range dequantises exactly like q8_dequantize_vec
        ko = torch.zeros(T * KV * hd, device="cuda")
        vo = torch.zeros_like(ko)
        kv.read_range(1, 0, T, ko.data_ptr(), vo.data_ptr())
        torch.cuda.synchronize()
        okv = oracle.kv_create(2, KV, hd, 64)
        try:
            for t in range(T):
                oracle.L.orc_kv_append(okv, 1, t, k[t].ctypes.data, v[t].ctypes.data)
            rk = np.zeros(T * KV * hd, np.float32)
            rv = np.zeros_like(rk)
            oracle.L.orc_kv_read_range(okv, 1, 0, T, rk.ctypes.data, rv.ctypes.data)
        finally:
            oracle.kv_destroy(okv)
        assert np.array_equal(ko.cpu().numpy(), rk) and np.array_equal(vo.cpu().numpy(), rv)
        kv.clear()
        assert kv.seq_len(1) == 0
    finally:
        kv.close()


@pytest.mark.parametrize("path", ["append", "append_range", "fused"])
def test_append_non_finite_like_the_reference(oracle, reference_q8, ctx, path):
    """NaN and +-inf inputs: the reference's maximum skips NaN (a > max_abs is
    false), an infinite maximum makes the scale inf, and (int)lrintf of NaN (NaN
    / scale, inf / inf) is 0 with the x86-64 C library (lrintf returns LONG_MIN,
    whose low 32 bits are 0); the GPU's round-to-nearest conversion gives 0 for
    NaN too.  Every appended block, scale and quants, must match byte for byte."""
    KV, hd, T = 2, 64, 6
    rng = np.random.default_rng(3)
    k = rng.normal(0, 1, (T, KV * hd)).astype(np.float32)
    v = rng.normal(0, 1, (T, KV * hd)).astype(np.float32)
    k[0, 3] = np.nan              # NaN among finite values
    k[1, 40] = np.inf             # +inf: scale inf, finite values quantise to 0
    v[2, 70] = -np.inf
    v[3, :32] = np.nan            # an all-NaN block
    k[4, 64:96] = np.inf          # an all-inf block
    v[5, 1] = np.nan
    v[5, 2] = np.inf
    kv = sc.KvCache(ctx, 1, KV, hd, 16)
    try:
        kd, vd = to_dev(k), to_dev(v)
        if path == "append":
            for t in range(T):
                kv.append(0, t, kd[t].data_ptr(), vd[t].data_ptr())
        elif path == "append_range":
            kv.append_range(0, 0, T, kd.data_ptr(), vd.data_ptr())
        else:  # the attention kernel's in-register quantiser (new row fused)
            q = to_dev(np.zeros(KV * hd, np.float32))
            out = torch.zeros(KV * hd, device="cuda")
            for t in range(T):
                kv.attend(0, q.data_ptr(), out.data_ptr(), KV, t + 1, 0.125, k_new=kd[t].data_ptr(),
                          v_new=vd[t].data_ptr())
        nb = KV * hd // 32 * 36
        kb = torch.zeros(T * nb, dtype=torch.uint8, device="cuda")
        vb = torch.zeros_like(kb)
        kv.read_blocks(0, 0, T, kb.data_ptr(), vb.data_ptr())
        torch.cuda.synchronize()
        ctx.check()
        for arr, got in ((k, kb), (v, vb)):
            want = np.concatenate([oracle.q8_quantize(arr[t]) for t in range(T)])
            assert np.array_equal(got.cpu().numpy(), want)
            if reference_q8 is not None:
                assert np.array_equal(want, np.concatenate([reference_q8(arr[t]) for t in range(T)]))
    finally:
        kv.close()


@pytest.fixture(scope="module")
def reference_q8():
    """The reference's own quantiser (oracle/_ref) when it is built here."""
    from oracle.oracle_py import Reference
    return Reference().q8_quantize if Reference.available() else None


@pytest.mark.parametrize("H,KV,hd", [(8, 2, 64), (32, 8, 128), (64, 8, 128), (4, 4, 128), (32, 4, 64),
                                     (8, 4, 128)])
@pytest.mark.parametrize("seq", [1, 2, 63, 64, 65, 300, 2049, 9001, 20000])  # >= 4096: split kernel
@pytest.mark.parametrize("new_row", ["fused", "pre_appended"])
def test_attend(oracle, ctx, H, KV, hd, seq, new_row):
    check_attend(oracle, ctx, H, KV, hd, seq, new_row, seq + 8)


@pytest.mark.parametrize("H,KV,hd", [(8, 2, 64), (64, 8, 128), (8, 1, 128)])
@pytest.mark.parametrize("seq", [1, 65, 300, 700, 4000])
def test_attend_long_cache(oracle, ctx, H, KV, hd, seq):
    """A cache of 8192 positions attends with the staged split kernel at
    every length: one cluster of splits (merged in distributed shared memory)
    up to 2048 positions, several clusters merged through global memory
    beyond; one KV head (a tensor-parallel rank of the 70B shape) included."""
    check_attend(oracle, ctx, H, KV, hd, seq, "fused", 8192)


@pytest.mark.parametrize("H,KV,hd,seq", [(64, 8, 128, 19531), (32, 8, 128, 19531), (8, 2, 64, 33789)])
@pytest.mark.parametrize("qscale", [1.0, 30.0])
def test_attend_tensor_core_ranges(oracle, ctx, H, KV, hd, seq, qscale):
    """Splits of 264 positions (more than the 256 that route a split to the
    tensor-core loop, not a multiple of its 16-position chunks: a masked last
    chunk), and queries 30x larger (scores near 100, a near one-hot
    softmax, where the three-part f16 split of q must keep fp32-level score
    error)."""
    check_attend(oracle, ctx, H, KV, hd, seq, "fused", seq + 9, qscale=qscale)


def check_attend(oracle, ctx, H, KV, hd, seq, new_row, cap, qscale=1.0):
    rng = np.random.default_rng(H * 131 + seq)
    k, v = kv_inputs(rng, seq, KV, hd)
    k[seq - 1, 5] = 3.0
    q = (rng.normal(0, 1, H * hd) * qscale).astype(np.float32)
    kv = sc.KvCache(ctx, 1, KV, hd, cap)
    try:
        kd, vd, qd = to_dev(k), to_dev(v), to_dev(q)
        n_pre = seq - 1 if new_row == "fused" else seq
        if n_pre:
            kv.append_range(0, 0, n_pre, kd.data_ptr(), vd.data_ptr())
        out = torch.zeros(H * hd, device="cuda")
        scale = np.float32(1.0 / np.sqrt(hd))
        if new_row == "fused":
            # the last position is quantised and appended by the attention kernel itself
            kv.attend(0, qd.data_ptr(), out.data_ptr(), H, seq, float(scale),
                      k_new=kd[seq - 1].data_ptr(), v_new=vd[seq - 1].data_ptr())
        else:
            kv.attend(0, qd.data_ptr(), out.data_ptr(), H, seq, float(scale))
        nb = KV * hd // 32 * 36
        kb = torch.zeros(nb, dtype=torch.uint8, device="cuda")
        vb = torch.zeros_like(kb)
        kv.read_blocks(0, seq - 1, seq, kb.data_ptr(), vb.data_ptr())
        torch.cuda.synchronize()
        ctx.check()
        got = out.cpu().numpy()
        assert np.array_equal(kb.cpu().numpy(), oracle.q8_quantize(k[seq - 1]))
        assert np.array_equal(vb.cpu().numpy(), oracle.q8_quantize(v[seq - 1]))
    finally:
        kv.close()
    okv = oracle.kv_create(1, KV, hd, seq + 8)
    try:
        for t in range(seq):
            oracle.L.orc_kv_append(okv, 0, t, k[t].ctypes.data, v[t].ctypes.data)
        K = np.zeros(seq * KV * hd, np.float32)
        V = np.zeros_like(K)
        oracle.L.orc_kv_read_range(okv, 0, 0, seq, K.ctypes.data, V.ctypes.data)
    finally:
        oracle.kv_destroy(okv)
    ref = oracle.attention(q, K, V, H, KV, hd, seq, scale)
    err = np.abs(got - ref).reshape(H, hd).max(axis=1)
    lim = 2e-5 * np.maximum(np.abs(ref).reshape(H, hd).max(axis=1), 1.0) + 8.0 * score_rounding_bound(
        q, K, V, H, KV, hd, seq, scale)
    assert np.all(err <= lim), (err / lim).max()


def score_rounding_bound(q, K, V, H, KV, hd, seq, scale):
    """Per head: the first-order effect on the output of fp32 rounding of the
    scores, u * sum_t p_t * S_t * max_d |V_td - out_d| with u = 2^-24 and S_t
    = scale * sum_d |q_d K_td| (in float64).  Two fp32 evaluations in
    different orders (the oracle's sequential dot products, the kernel's
    per-block sums) differ by a few times this; it is negligible for
    well-spread softmaxes and dominates when large queries make the softmax
    near one-hot (the oracle itself is then ~2x this away from the exact
    value)."""
    K3 = K.reshape(seq, KV, hd).astype(np.float64)
    V3 = V.reshape(seq, KV, hd).astype(np.float64)
    Q = q.reshape(H, hd).astype(np.float64)
    out = np.empty(H)
    for h in range(H):
        kvh = h % KV
        s = K3[:, kvh, :] @ Q[h] * float(scale)
        sa = np.abs(K3[:, kvh, :]) @ np.abs(Q[h]) * float(scale)
        p = np.exp(s - s.max())
        p /= p.sum()
        dev = np.abs(V3[:, kvh, :] - p @ V3[:, kvh, :]).max(axis=1)
        out[h] = (p * sa * dev).sum() * 2.0**-24
    return out


@pytest.mark.parametrize("H,KV,hd,seq", [(64, 8, 128, 300), (64, 8, 128, 5000), (8, 2, 64, 1500),
                                          (8, 4, 64, 4200), (4, 4, 128, 9000)])
def test_attend_batch(oracle, ctx, H, KV, hd, seq):
    """Three sequences (cache layers 1..3) in one launch: each appends its new
    row bit-exactly and attends as the oracle does on its own K/V."""
    B = 3
    rng = np.random.default_rng(H * 7 + seq)
    kv = sc.KvCache(ctx, B + 1, KV, hd, seq + 16)
    try:
        ks, vs, keep = [], [], []
        for b in range(B):
            k, v = kv_inputs(rng, seq, KV, hd)
            k[seq - 1, 5] = 3.0
            ks.append(k)
            vs.append(v)
            keep += [to_dev(k), to_dev(v)]  # alive until the appends have run
            kv.append_range(1 + b, 0, seq - 1, keep[-2].data_ptr(), keep[-1].data_ptr())
        q = (rng.normal(0, 1, (B, H * hd))).astype(np.float32)
        kn = np.stack([k[seq - 1] for k in ks])
        vn = np.stack([v[seq - 1] for v in vs])
        qd, knd, vnd = to_dev(q), to_dev(kn), to_dev(vn)
        out = torch.zeros(B, H * hd, device="cuda")
        scale = np.float32(1.0 / np.sqrt(hd))
        kv.attend_batch(1, B, qd.data_ptr(), out.data_ptr(), H, seq, float(scale), knd.data_ptr(), vnd.data_ptr())
        torch.cuda.synchronize()
        ctx.check()
        got = out.cpu().numpy()
        nb = KV * hd // 32 * 36
        for b in range(B):
            kb = torch.zeros(nb, dtype=torch.uint8, device="cuda")
            vb = torch.zeros_like(kb)
            kv.read_blocks(1 + b, seq - 1, seq, kb.data_ptr(), vb.data_ptr())
            torch.cuda.synchronize()
            assert np.array_equal(kb.cpu().numpy(), oracle.q8_quantize(ks[b][seq - 1]))
            assert np.array_equal(vb.cpu().numpy(), oracle.q8_quantize(vs[b][seq - 1]))
            assert kv.seq_len(1 + b) == seq
    finally:
        kv.close()
    for b in range(B):
        okv = oracle.kv_create(1, KV, hd, seq + 8)
        try:
            for t in range(seq):
                oracle.L.orc_kv_append(okv, 0, t, ks[b][t].ctypes.data, vs[b][t].ctypes.data)
            K = np.zeros(seq * KV * hd, np.float32)
            V = np.zeros_like(K)
            oracle.L.orc_kv_read_range(okv, 0, 0, seq, K.ctypes.data, V.ctypes.data)
        finally:
            oracle.kv_destroy(okv)
        ref = oracle.attention(q[b], K, V, H, KV, hd, seq, scale)
        err = np.abs(got[b] - ref).reshape(H, hd).max(axis=1)
        lim = 2e-5 * np.maximum(np.abs(ref).reshape(H, hd).max(axis=1), 1.0) + 8.0 * score_rounding_bound(
            q[b], K, V, H, KV, hd, seq, scale)
        assert np.all(err <= lim), (b, (err / lim).max())


def test_attend_rejects_out_of_range(ctx):
    kv = sc.KvCache(ctx, 1, 2, 64, 16)
    try:
        q = torch.zeros(4 * 64, device="cuda")
        with pytest.raises(sc.ShkError):
            kv.attend(0, q.data_ptr(), q.data_ptr(), 4, 17, 0.125)
    finally:
        kv.close()

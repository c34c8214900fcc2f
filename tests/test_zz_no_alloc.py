"""shk_cuda_argmax_noalloc -- the argmax for callers that cannot allocate
device memory (its scratch is a fixed array inside the library) -- against
the context-based shk_cuda_argmax, through the C ABI.

Two calls in a row on different inputs: the second must not see the first
call's partials, since every call shares the same fixed scratch array.  The
file is named to be collected last; it needs nothing from earlier tests.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from shukuchi_b200 import cuda as sc

pytestmark = pytest.mark.gpu


def _noalloc(x_dev, n):
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = sc.lib().shk_cuda_argmax_noalloc(x_dev.data_ptr(), n, out.data_ptr(), stream)
    assert rc == sc.SHK_OK, sc.STATUS.get(rc, rc)
    torch.cuda.synchronize()
    return int(out.cpu().numpy().view(np.uint32)[0])


def test_argmax_noalloc_matches_argmax():
    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    torch.cuda.set_device(0)
    ctx = sc.Context(0)
    try:
        rng = np.random.default_rng(2024)
        # vocabulary-sized (148 blocks) then a small one (1 block), max moved
        for n, where in ((128256, (77777, 100001)), (1000, (5, 999))):
            x = rng.normal(0, 1, n).astype(np.float32)
            x[list(where)] = x.max() + 1.0  # a tie: the first index must win
            xd = torch.from_numpy(x).cuda()
            got = _noalloc(xd, n)
            want = ctx.argmax(xd.data_ptr(), n)
            assert got == want == where[0], (n, got, want)
    finally:
        ctx.close()


def test_argmax_noalloc_last_partial_block():
    # n spans several 4096-element argmax blocks with a short last one; the
    # maximum sits in that last partial block, then at its very last element
    rng = np.random.default_rng(7)
    n = 3 * 4096 + 100
    x = rng.normal(0, 1, n).astype(np.float32)
    for where in (3 * 4096 + 37, n - 1):
        y = x.copy()
        y[where] = 10.0
        got = _noalloc(torch.from_numpy(y).cuda(), n)
        assert got == where, (got, where)


def test_argmax_noalloc_rejects_bad_sizes():
    lib = sc.lib()
    x = torch.zeros(4, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.shk_cuda_argmax_noalloc(x.data_ptr(), 0, out.data_ptr(), None) == -1
    # one past the largest accepted n (SHK_ARGMAX_NOALLOC_MAX_N = 0xFFFFFFFE)
    assert lib.shk_cuda_argmax_noalloc(x.data_ptr(), 0xFFFFFFFE + 1, out.data_ptr(), None) == -1
    assert lib.shk_cuda_argmax_noalloc(None, 4, out.data_ptr(), None) == -1
    assert int(out.cpu()[0]) == 0  # nothing was launched
    # the context-based argmax takes the same bound
    ctx = sc.Context(0)
    try:
        res = C.c_uint32(7)
        assert lib.shk_cuda_argmax(ctx.h, x.data_ptr(), 0xFFFFFFFE + 1, C.byref(res)) == -1
        assert res.value == 7
    finally:
        ctx.close()

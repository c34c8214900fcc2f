import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libshk_cuda.so")
    config.addinivalue_line("markers", "slow: large model shapes")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle_py import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle_py import Reference
    if not Reference.available():
        pytest.skip("reference build (oracle/_ref) not present on this machine")
    return Reference()


def golden(name: str):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


@pytest.fixture(scope="session")
def ctx():
    import torch
    from shukuchi_b200 import cuda as sc
    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    torch.cuda.init()
    c = sc.Context(0)
    yield c
    c.close()


def to_dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gemv_tolerance(oracle, qtype, w, x, m, k):
    """Per-row bound: 4*sqrt(k)*2^-24 times the L1 mass sum_k |w_rk * x_k|
    (fp32 summation in two different orders), plus a tiny absolute floor."""
    bb = {12: 144, 13: 176, 14: 210}[qtype]
    rowb = (k // 256) * bb
    W = np.stack([oracle.dequant(qtype, w[r * rowb:(r + 1) * rowb], k) for r in range(m)])
    mass = np.abs(W) @ np.abs(x.astype(np.float64))
    return 4.0 * np.sqrt(k) * 2.0 ** -24 * mass + 1e-30

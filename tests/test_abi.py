"""CPU-side checks of the drop-in boundary: the library loads without a GPU and
exports every function include/shk_cuda.h declares; the ctypes mirror covers
the same set."""
import ctypes
import os

import pytest

from shukuchi_b200 import cuda as sc


def test_header_functions_exported():
    if not os.path.exists(sc.LIB_PATH):
        pytest.fail("libshk_cuda.so not built (python -m shukuchi_b200.build)")
    L = ctypes.CDLL(sc.LIB_PATH)
    names = sc.header_functions()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_ctypes_mirror_matches_header():
    assert set(sc.header_functions()) == set(sc._SIGS)


def test_status_strings():
    L = sc.lib()
    assert L.shk_cuda_strerror(-5) == b"bounded device wait ran out"
    assert L.shk_cuda_strerror(0) == b"ok"


def test_available_reports_no_device_on_cpu_box():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert sc.lib().shk_cuda_available() == 0
    # init must refuse rather than fall back to anything
    assert not sc.lib().shk_cuda_init(None)

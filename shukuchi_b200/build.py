"""Builds the in-tree native libraries.

* ``shukuchi_b200/libshk_cuda.so`` -- every CUDA kernel plus the C ABI of
  ``include/shk_cuda.h``, compiled for sm_100a only.
* ``shukuchi_b200/engine/libshukuchi.so`` and the ``shukuchi`` CLI -- the C
  engine (GGUF reader, loader, prefetcher, decode loop) over that ABI.

Run ``python -m shukuchi_b200.build`` (or ``__graft_entry__.build()``).  Objects
are compiled in parallel and cached by source mtime under ``_build/``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
ENGINE = os.path.join(PKG, "engine")
BUILD = os.path.join(ROOT, "_build")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-I" + os.path.join(ROOT, "include")]
CUDA_LIB = os.path.join(os.path.dirname(os.path.dirname(NVCC)), "lib64")
LIB = os.path.join(PKG, "libshk_cuda.so")


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers(d: str) -> list[str]:
    return [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".cuh", ".h"))]


def build_cuda(verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    hdrs = _headers(CSRC) + [os.path.join(ROOT, "include", "shk_cuda.h")]
    objs = []
    jobs = []
    for s in srcs:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace(".cu", ".o"))
        objs.append(obj)
        if _stale(obj, [src] + hdrs) or verbose_ptxas:
            extra = ["-Xptxas", "-v"] if verbose_ptxas else []
            jobs.append(NVCC_FLAGS + extra + ["-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        for f in [ex.submit(_run, [NVCC] + j) for j in jobs]:
            f.result()
    if _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-lpthread", "-ldl"])
    return LIB


def build_engine() -> str | None:
    """Builds the C engine library and CLI if their sources exist."""
    srcs = sorted(os.path.join(ENGINE, f) for f in os.listdir(ENGINE) if f.endswith(".c")) \
        if os.path.isdir(ENGINE) else []
    if not srcs:
        return None
    lib = os.path.join(ENGINE, "libshukuchi.so")
    cli = os.path.join(ENGINE, "shukuchi")
    lib_srcs = [s for s in srcs if not s.endswith("main.c")]
    hdrs = _headers(ENGINE) + [os.path.join(ROOT, "include", "shk_cuda.h")]
    cflags = ["-std=c11", "-D_GNU_SOURCE", "-O2", "-fPIC", "-Wall", "-I" + ENGINE,
              "-I" + os.path.join(ROOT, "include")]
    if _stale(lib, lib_srcs + hdrs + [LIB]):
        _run(["gcc"] + cflags + ["-shared", "-o", lib] + lib_srcs +
             ["-L" + PKG, "-lshk_cuda", "-Wl,-rpath,$ORIGIN/..", "-lpthread", "-lm"])
    packer_dir = os.path.join(PKG, "packer")
    if os.path.isdir(packer_dir):  # the LSTR packer CLI (GGUF -> container)
        psrcs = [os.path.join(packer_dir, f) for f in ("packer.c", "main.c")] + \
                [os.path.join(ENGINE, f) for f in ("gguf.c", "lstr.c")]
        pbin = os.path.join(packer_dir, "shukuchi-pack")
        if _stale(pbin, psrcs + hdrs + _headers(packer_dir)):
            _run(["gcc"] + cflags + ["-o", pbin] + psrcs)
    main = os.path.join(ENGINE, "main.c")
    if os.path.exists(main) and _stale(cli, [main, lib]):
        _run(["gcc"] + cflags + ["-o", cli, main, "-L" + ENGINE, "-lshukuchi",
                                 "-Wl,-rpath,$ORIGIN", "-Wl,-rpath,$ORIGIN/.."])
    return lib


def build_oracle() -> None:
    """Compiles the oracle: oracle/liboracle.so always, oracle/_ref when the
    reference sources are present on this machine."""
    od = os.path.join(ROOT, "oracle")
    _run(["make", "-s", "-C", od, "liboracle.so"])
    # the Makefile knows where the reference sources are (and whether they are)
    if subprocess.run(["make", "-s", "-C", od, "ref-present"], capture_output=True).returncode == 0:
        _run(["make", "-s", "-C", od, "ref"])


def build_all(verbose_ptxas: bool = False) -> None:
    build_cuda(verbose_ptxas)
    build_engine()
    build_oracle()


if __name__ == "__main__":
    build_all(verbose_ptxas="-v" in sys.argv)
    print("built", LIB)

"""Builds the sm_100a shared library ``bee_b200/_lib/libbee_b200.so``.

All CUDA sources under ``bee_b200/csrc`` plus the C++ host bridge under
``bee_b200/host`` are compiled by nvcc for ``sm_100a`` only and linked into one
shared object that exports the C ABI declared in ``include/bee_b200.h``.  The
CUDA runtime is linked statically, so the library only needs the driver
(``libcuda.so``) at run time; the driver entry point for tensor-map encoding
is looked up through ``cudaGetDriverEntryPoint``.

Usage: ``python -m bee_b200.build [--force]``.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libbee_b200.so"
OBJ_DIR = PKG / "_lib" / "obj"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(ROOT / "include"),
    "-DBEE_B200_BUILD",
]
CUDA_INC = str(Path(NVCC).resolve().parent.parent / "include")
HOST_FLAGS = ["-O2", "-std=c++23", "-fPIC", "-I", str(ROOT / "include"), "-I", str(HOST), "-I", CUDA_INC]
HOST_TEST_SRC = ROOT / "tests" / "cpp" / "test_host_bridge.cpp"
HOST_TEST_BIN = LIB_DIR / "test_host_bridge"
BRIDGE_BENCH_SRC = HOST / "bridge_bench.cpp"
BRIDGE_BENCH_BIN = LIB_DIR / "bridge_bench"


def _sources():
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted(p for p in HOST.glob("*.cpp") if p.name != "bridge_bench.cpp")  # a program, not library code
    headers = sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h")) + sorted(HOST.glob("*.hpp"))
    return cu, cpp, headers


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(map(str, cmd)) + "\n" + r.stdout)
        raise RuntimeError(f"build step failed ({r.returncode}): {cmd[0]} {cmd[-1]}")
    return r.stdout


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every source that changed and relinks the library; returns its path."""
    cu, cpp, headers = _sources()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    for src in cu:
        obj = OBJ_DIR / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            out = _run([NVCC, *ARCH, *NVCC_FLAGS, "-Xptxas", "-v", "-c", str(src), "-o", str(obj)]
                       if verbose else [NVCC, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
            if verbose:
                sys.stdout.write(out)
        objs.append(obj)
    for src in cpp:
        obj = OBJ_DIR / (src.stem + ".host.o")
        if force or _stale(obj, [src] + headers):
            _run(["g++", *HOST_FLAGS, "-c", str(src), "-o", str(obj)])
        objs.append(obj)
    if force or _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lrt", "-ldl", "-lpthread"])
    # C++ program exercising the host bridge (run by tests/test_gpu_host_bridge.py)
    if HOST_TEST_SRC.exists() and (force or _stale(HOST_TEST_BIN, [HOST_TEST_SRC, LIB] + headers)):
        _run(["g++", *HOST_FLAGS, str(HOST_TEST_SRC), "-o", str(HOST_TEST_BIN), "-L", str(LIB_DIR), "-lbee_b200",
              "-Wl,-rpath,$ORIGIN"])
    # measurement program for the bridge's plumbing cost (run by bench.py)
    if BRIDGE_BENCH_SRC.exists() and (force or _stale(BRIDGE_BENCH_BIN, [BRIDGE_BENCH_SRC, LIB] + headers)):
        _run(["g++", *HOST_FLAGS, str(BRIDGE_BENCH_SRC), "-o", str(BRIDGE_BENCH_BIN), "-L", str(LIB_DIR),
              "-lbee_b200", "-Wl,-rpath,$ORIGIN"])
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()

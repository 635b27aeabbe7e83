"""Build recipe for the native parts of powersparse_b200 (in-tree, sm_100a).

    python -m powersparse_b200.build           # everything
    python -m powersparse_b200.build cuda      # libpowersparse_b200.so only

Outputs (git-ignored, shipped with the tree):
  powersparse_b200/lib/libpowersparse_b200.so  C ABI + CUDA kernels (include/powersparse_b200.h)
  powersparse_b200/lib/libpowersparse_b200_checked.so   the same with bounds-checked kernels
  powersparse_b200/lib/libpowersparse.so       the reference's C++ operator API over the C ABI
  powersparse_b200/bin/powersparse_spmm        drop-in benchmark CLI (SpMM)
  powersparse_b200/bin/powersparse_sddmm       drop-in benchmark CLI (SDDMM)
  powersparse_b200/bin/powersparse_mtx2csr     MatrixMarket -> binary CSR converter
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "lib")
BIN = os.path.join(PKG, "bin")
INCLUDE = os.path.join(ROOT, "include")

NVCC = os.environ.get("NVCC", "nvcc")
HOSTCXX = os.environ.get("PS_HOSTCXX", "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_LIBDIR = os.path.join(os.path.dirname(os.path.dirname(os.path.realpath(
    subprocess.run(["which", NVCC], capture_output=True, text=True).stdout.strip() or "/usr/local/cuda/bin/nvcc"))),
    "lib64")

CUDA_LIB = os.path.join(LIB, "libpowersparse_b200.so")
# The same library with every operator kernel checking the indices it follows
# (-DPSB_BOUNDS_CHECK; see ps_ops.cu).  For debugging: each operator call waits for
# its kernels.  Load it with PSB_LIBRARY=<path> (powersparse_b200.load_library).
CHECKED_LIB = os.path.join(LIB, "libpowersparse_b200_checked.so")
CXX_LIB = os.path.join(LIB, "libpowersparse.so")


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd[:4]) + " ...")


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_cuda(force: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = srcs + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        [os.path.join(INCLUDE, "powersparse_b200.h")]
    os.makedirs(LIB, exist_ok=True)
    for target, flags in ((CUDA_LIB, []), (CHECKED_LIB, ["-DPSB_BOUNDS_CHECK=1"])):
        if force or _stale(target, deps):
            _run([NVCC, "-std=c++17", "-O3", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-shared", *flags,
                  "-ccbin", HOSTCXX, "-I" + INCLUDE, "-o", target, *srcs])
    return CUDA_LIB


def build_cxx(force: bool = False) -> None:
    """The reference's C++ API (namespace PowerSparse) and the drop-in CLI."""
    host = sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    reader = [os.path.join(CSRC, "cli", "matrix_market.cpp")]
    cli = [os.path.join(CSRC, "cli", "benchmark.cpp")] + reader
    convert = [os.path.join(CSRC, "cli", "mtx2csr.cpp")] + reader
    if not host:
        return
    hdrs = glob.glob(os.path.join(INCLUDE, "**", "*.h"), recursive=True)
    cuda_inc = os.path.join(os.path.dirname(CUDA_LIBDIR), "include")
    common = ["-std=c++17", "-O2", "-I" + INCLUDE, "-I" + cuda_inc]
    if force or _stale(CXX_LIB, host + hdrs + [CUDA_LIB]):
        _run([HOSTCXX, *common, "-fPIC", "-shared", "-o", CXX_LIB, *host, "-L" + LIB, "-lpowersparse_b200",
              "-L" + CUDA_LIBDIR, "-lcudart", "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + CUDA_LIBDIR])
    cli_hdrs = hdrs + [os.path.join(CSRC, "cli", "matrix_market.h")]
    os.makedirs(BIN, exist_ok=True)
    for op, define in (("spmm", []), ("sddmm", ["-DPOWERSPARSE_BENCH_SDDMM=1"])):
        target = os.path.join(BIN, f"powersparse_{op}")
        if force or _stale(target, cli + cli_hdrs + [CXX_LIB]):
            _run([HOSTCXX, *common, "-O3", "-pthread", *define, "-o", target, *cli, "-L" + LIB, "-lpowersparse",
                  "-lpowersparse_b200", "-L" + CUDA_LIBDIR, "-lcudart",
                  "-Wl,-rpath,$ORIGIN/../lib", "-Wl,-rpath," + CUDA_LIBDIR])
    # MatrixMarket -> binary CSR converter (host only, no CUDA).
    target = os.path.join(BIN, "powersparse_mtx2csr")
    if force or _stale(target, convert + cli_hdrs):
        _run([HOSTCXX, "-std=c++17", "-O3", "-pthread", "-o", target, *convert])


def build_all(force: bool = False) -> None:
    build_cuda(force)
    build_cxx(force)


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    if what == "cuda":
        build_cuda(force=True)
    else:
        build_all(force=True)
    print("built", CUDA_LIB)

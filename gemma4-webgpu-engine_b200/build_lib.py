"""Build libgemma4_cuda.so in-tree with nvcc for sm_100a (B200).

The library is the product: every kernel, the executor and the C ABI declared in
include/g4.h. It is compiled with --fmad=false (fused multiply-adds only where the source calls
fmaf) and IEEE division and square root, the arithmetic contract the kernels are written to.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libgemma4_cuda.so"
SOURCES = ["g4_kernels.cu", "g4_gemv2.cu", "g4_gemm.cu", "g4_ple.cu", "g4_runtime.cu", "g4_noalloc.cu"]
HEADERS = ["g4_device.cuh", "g4_kernels.cuh", "g4_gemv.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "--fmad=false", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent / "include" / "g4.h", Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


TRACE_LIB = LIB_DIR / "trace" / "libgemma4_cuda.so"
NAPI_SRC = PKG / "napi" / "g4_napi.c"
NAPI_ADDON = LIB_DIR / "gemma4_cuda.node"


def build_napi(verbose: bool = False) -> Path:
    """The Node-API addon (gemma4_cuda.node) over libgemma4_cuda.so. Node's napi_* symbols stay
    undefined until Node (or another Node-API host) loads the addon."""
    if NAPI_ADDON.exists() and NAPI_ADDON.stat().st_mtime > max(
            NAPI_SRC.stat().st_mtime, LIB.stat().st_mtime, (PKG / "napi" / "node_api_min.h").stat().st_mtime):
        return NAPI_ADDON
    cmd = [os.environ.get("CC", "gcc"), "-O2", "-std=c11", "-fPIC", "-shared", "-Wall", "-Wextra",
           "-Wno-unused-parameter", str(NAPI_SRC), "-o", str(NAPI_ADDON), f"-L{LIB_DIR}",
           "-lgemma4_cuda", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return NAPI_ADDON


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> Path:
    """Build the library (or, with trace=True, the diagnostic build with kernel time stamps
    into lib/trace/, which the `trace` module reads; never the library the package loads)."""
    out = TRACE_LIB if trace else LIB
    if not force and not trace and not needs_build():
        return LIB
    out.parent.mkdir(parents=True, exist_ok=True)
    objs, procs = [], []
    extra = ["-DG4_TRACE"] if trace else []
    for src in SOURCES:   # the translation units compile in parallel
        obj = out.parent / (Path(src).stem + ".o")
        cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((subprocess.Popen(cmd), cmd))
        objs.append(str(obj))
    failed = [cmd for p, cmd in procs if p.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    tmp = out.with_suffix(".so.tmp")
    cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    for o in objs:
        Path(o).unlink(missing_ok=True)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, trace="--trace" in sys.argv))
    if "--trace" not in sys.argv:
        print(build_napi(verbose=True))

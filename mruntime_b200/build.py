"""Build the sm_100a shared library in-tree: mruntime_b200/_build/libmrt_b200.so.

Every .cu under csrc/ is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked with the static
CUDA runtime, so the library loads on hosts without a GPU driver (the
driver is reached through cudaGetDriverEntryPoint at run time).  NCCL is
opened with dlopen by the library itself; only its header is needed here.

When the reference's headers are present, the C++ ``CudaBackend`` (a
``mruntime::Backend``) is also built as _build/libmrt_cuda_backend.so.

    python -m mruntime_b200.build            # build what is out of date
    python -m mruntime_b200.build --force    # rebuild everything
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(BUILD, "libmrt_b200.so")
BACKEND_LIB = os.path.join(BUILD, "libmrt_cuda_backend.so")
INCLUDE = os.path.join(ROOT, "include")
REFERENCE_INCLUDE = os.environ.get("MRT_REFERENCE_INCLUDE", "/root/reference/include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", "-Xptxas", "-v"]

KERNEL_SOURCES = ["capi.cu", "tp.cu", "gemm_tc.cu", "gemv.cu", "elementwise.cu", "general_gemm.cu", "ops.cu", "noalloc.cu",
                  "decoder.cu", "decode_step.cu", "loader.cu"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _nccl_include() -> list[str]:
    try:
        import nvidia.nccl  # type: ignore
        inc = os.path.join(os.path.dirname(nvidia.nccl.__file__), "include")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return ["-I" + inc]
    except Exception:
        pass
    return []


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs + [os.path.join(INCLUDE, "mrt_b200.h")]


def _compile(src: str, obj: str, log_dir: str) -> str:
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-I" + INCLUDE, "-I" + CSRC, *_nccl_include(), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    with open(os.path.join(log_dir, os.path.basename(src) + ".ptxas.txt"), "w") as f:
        f.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr[-6000:]}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    jobs = []
    hdrs = _headers()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for name in KERNEL_SOURCES:
            src = os.path.join(CSRC, name)
            obj = os.path.join(BUILD, name.replace(".cu", ".o"))
            objs.append(obj)
            if force or _stale(obj, [src, *hdrs]):
                jobs.append(ex.submit(_compile, src, obj, BUILD))
        for j in jobs:
            j.result()
    if force or jobs or _stale(LIB, objs):
        cmd = [_nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    if verbose:
        print(LIB)
    build_backend(force=force, verbose=verbose)
    return LIB


def build_backend(force: bool = False, verbose: bool = False) -> str | None:
    """C++ CudaBackend against the reference's Backend interface (its header is
    included where it lies, not copied).  Skipped when the headers are absent."""
    src = os.path.join(CSRC, "cuda_backend.cpp")
    hdr = os.path.join(CSRC, "cuda_backend.h")
    if not os.path.exists(src) or not os.path.exists(os.path.join(REFERENCE_INCLUDE, "mruntime", "backend.h")):
        return None
    if not (force or _stale(BACKEND_LIB, [src, hdr, LIB])):
        return BACKEND_LIB
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-I" + INCLUDE, "-I" + CSRC,
           "-I" + REFERENCE_INCLUDE, "-I/usr/local/cuda/include", src, "-o", BACKEND_LIB,
           "-L" + BUILD, "-lmrt_b200", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"CudaBackend build failed:\n{r.stderr[-4000:]}")
    if verbose:
        print(BACKEND_LIB)
    return BACKEND_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    try:
        build(force=args.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)

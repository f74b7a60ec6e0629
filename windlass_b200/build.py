"""Builds libwindlass_cuda.so in-tree with nvcc for sm_100a (no PyTorch, no JIT cache).

    python -m windlass_b200.build          # or: python windlass_b200/build.py

Objects go to _build/ (not committed); the library lands next to this file, where windlass_b200/_lib.py loads it.
Every source is compiled with -gencode arch=compute_100a,code=sm_100a -lineinfo, CUDA runtime linked statically,
NCCL loaded at run time (dlopen) by the tensor-parallel paths only.
"""
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libwindlass_cuda.so")

SOURCES = ["wl_kernels.cu", "wl_mmv.cu", "wl_mmv_i8.cu", "wl_noalloc.cu", "wl_model.cpp", "wl_gguf.cpp", "wl_common.cpp", "wl_api.cpp",
           "wl_nccl.cpp", "wl_stream.cpp", "wl_gemm.cu", "wl_group.cpp", "wl_sample.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    deps.append(os.path.join(ROOT, "include", "windlass.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [nvcc(), "-c", path, "-o", obj, "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-Wall,-Wno-unused-function",
           "-I", os.path.join(ROOT, "include"), "-I", CSRC] + ARCH
    if src.endswith(".cu"):
        cmd += ["-Xptxas", "-warn-spills", "--expt-relaxed-constexpr"]
        if verbose:
            cmd += ["-Xptxas", "-v"]
    else:
        cmd = [c if c != "-c" else "-c" for c in cmd] + ["-x", "c++"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [nvcc(), "-shared", "-o", LIB] + objs + ARCH + ["-cudart", "static", "-lpthread", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))

"""Build libcbmoe.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python kaggle-llm-endpoint_b200/build.py          # -> kaggle-llm-endpoint_b200/cbmoe/libcbmoe.so

Every .cu under csrc/ is compiled with relocatable device code (one device symbol, the error word, is shared
across files) and linked into one shared library with the CUDA runtime linked statically. Objects go to
_build/ next to this file; a file is recompiled when it or any header under csrc/ or include/ is newer.
"""
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "cbmoe", "libcbmoe.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                "-I", INCLUDE, "-I", CSRC]


def _newest_header():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src, extra, verbose):
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _newest_header()):
        return obj
    cmd = [NVCC] + FLAGS + extra + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr, flush=True)
    return obj


def nccl_paths():
    """(include dir, lib dir) of the NCCL that torch bundles (nvidia-nccl wheel), or the system one."""
    try:
        import nvidia.nccl as nn
        base = os.path.dirname(nn.__file__) if getattr(nn, "__file__", None) else list(nn.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def build(verbose=False, ptxas_verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    nccl_inc, nccl_lib = nccl_paths()
    extra = ["-I", nccl_inc] + (["-Xptxas", "-v"] if ptxas_verbose else [])
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, verbose or ptxas_verbose), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    nccl_so = sorted(glob.glob(os.path.join(nccl_lib, "libnccl.so*")))
    link_nccl = ["-L", nccl_lib, "-Xlinker", f"-rpath={nccl_lib}", "-l:" + os.path.basename(nccl_so[0])] if nccl_so else []
    cmd = [NVCC] + ARCH + ["-shared", "-rdc=true", "-o", LIB] + objs + link_nccl
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_verbose="-v" in sys.argv))

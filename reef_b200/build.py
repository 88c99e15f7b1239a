"""Build libreef_b200.so in-tree with nvcc for sm_100a.

    python -m reef_b200.build [--force]

Every .cu / .cpp under reef_b200/csrc is compiled to reef_b200/_build/*.o with
``-gencode arch=compute_100a,code=sm_100a -lineinfo`` and linked into
reef_b200/libreef_b200.so (static CUDA runtime; NCCL from the wheel torch
ships, resolved by soname at load time).  Objects are rebuilt when their
source, any header or this file's flags are newer.  No fast-math: the W8A8
epilogues and the exact float kernels depend on IEEE rounding.  -fmad=false
keeps nvcc from contracting multiply-adds where a result is defined bit for
bit: reef's operators, the RMSNorm order and the RoPE / SwiGLU values that a
fused epilogue must reproduce (flash_attn.cu holds the unfused RoPE packing
the QKV epilogue matches bit for bit).  The decode head, checked within a
tolerance (FMA_FREE_EXEMPT), keeps nvcc's contraction.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libreef_b200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
          f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"]
# translation units whose float results are checked within a tolerance, not
# bit for bit: nvcc may contract their multiply-adds
FMA_FREE_EXEMPT = {"decode_attn.cu"}


def _nccl_dirs():
    """(include, lib) of the NCCL that torch loads (nvidia-nccl wheel)."""
    try:
        import nvidia.nccl as nn  # type: ignore
        base = list(nn.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h")) + [os.path.abspath(__file__)]


def _stale(src: str, obj: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(src: str, obj: str, nccl_inc: str, verbose: bool) -> str:
    fmad = [] if os.path.basename(src) in FMA_FREE_EXEMPT else ["-fmad=false"]
    cmd = [NVCC, *ARCH, *COMMON, *fmad, f"-I{nccl_inc}", "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd.insert(1, "-x")
        cmd.insert(2, "cu")
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return (r.stdout + r.stderr).strip()


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) +
                     glob.glob(os.path.join(CSRC, "*.cpp")))
    newest = max([os.path.getmtime(h) for h in _headers()] + [0.0])
    nccl_inc, nccl_lib = _nccl_dirs()
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(OUT_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or verbose or _stale(src, obj, newest):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, nccl_inc, verbose): s for s, o in jobs}
            for f in cf.as_completed(futs):
                msg = f.result()
                if verbose and msg:
                    print(f"== {os.path.basename(futs[f])}\n{msg}")
    lib_time = os.path.getmtime(LIB) if os.path.exists(LIB) else -1
    if jobs or lib_time < max(os.path.getmtime(o) for o in objs):
        # the wheel ships only libnccl.so.2, so name it exactly
        link = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, f"-L{nccl_lib}",
                "-Xlinker", "-l:libnccl.so.2", f"-Xlinker=-rpath,{nccl_lib}"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true",
                    help="rebuild with -Xptxas -v and print register/smem use")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())

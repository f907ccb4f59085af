"""Build recipe of the B200 path (in-tree; the built .so files travel with the repo).

  libspb200.so     sm_100a kernels + runtime + C ABI (include/spb200.h)   -- nvcc
  libspb200_l1.so  section-6/6b binding to the reference's L1 ABI          -- gcc,
                   compiled against the reference's own headers
                   (SPB_REF_INCLUDE; default: the `reference` tree beside this
                   repository, <repo>/../reference/include); skipped, with a
                   note, when those headers are absent.

Run: python shannon-prime-system_b200/build.py [--force]
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
CORE_SO = os.path.join(HERE, "libspb200.so")
L1_SO = os.path.join(HERE, "libspb200_l1.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
REF_INCLUDE = os.environ.get("SPB_REF_INCLUDE",
                             os.path.join(os.path.dirname(ROOT), "reference", "include"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"] + ARCH
CU_SRCS = ["spb_kernels.cu", "spb_gemm_tc.cu", "spb_runtime.cu", "spb_noalloc.cu", "spb_tp.cu"]
HDRS = ["spb_exact.cuh", "spb_kernels.cuh", "spb_async.cuh", "spb_device.cuh", "spb_tp.cuh", "spb_spinor.cuh"]


def _newer(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build(force: bool = False, verbose: bool = False) -> dict:
    os.makedirs(OBJ, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HDRS] + [os.path.join(ROOT, "include", "spb200.h")]
    objs = []
    jobs = []
    for src in CU_SRCS:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            jobs.append([NVCC] + NVFLAGS + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=4) as ex:
        list(ex.map(lambda c: _run(c, verbose), jobs))
    if force or jobs or _newer(CORE_SO, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", CORE_SO] + objs + ["-lcudart", "-ldl"], verbose)
    out = {"core": CORE_SO, "l1": None}
    l1_src = os.path.join(CSRC, "spb_l1.c")
    if os.path.exists(os.path.join(REF_INCLUDE, "sp", "sp_l1.h")):
        deps = [l1_src, CORE_SO, os.path.join(ROOT, "include", "spb200_l1.h")]
        if force or _newer(L1_SO, deps):
            _run(["gcc", "-std=c11", "-O2", "-fPIC", "-shared", "-Wall", "-I", REF_INCLUDE,
                  "-o", L1_SO, l1_src, "-L", HERE, "-lspb200", "-Wl,-rpath,$ORIGIN", "-lpthread"],
                 verbose)
        out["l1"] = L1_SO
    elif os.path.exists(L1_SO):
        out["l1"] = L1_SO
    else:
        print(f"note: {REF_INCLUDE}/sp/sp_l1.h not found; libspb200_l1.so not built", file=sys.stderr)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

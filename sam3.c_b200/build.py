"""Build recipe of libsam3cu.so (the B200 backend) for sm_100a.

    python sam3.c_b200/build.py          # incremental
    python sam3.c_b200/build.py --clean

Every .cu/.c under csrc/ is compiled by nvcc for `-gencode
arch=compute_100a,code=sm_100a` and linked into lib/libsam3cu.so, in tree,
so that the built library travels with the repository snapshot.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
# SAM3CU_BUILD_OUT=<dir> builds a variant library (<dir>/libsam3cu.so, objects
# in <dir>/_build) with the extra -D flags of SAM3CU_BUILD_DEFS, for A/B
# measurements of compile-time kernel switches (loaded via SAM3CU_LIB).
_VAR = os.environ.get("SAM3CU_BUILD_OUT")
OBJ = os.path.join(_VAR, "_build") if _VAR else os.path.join(HERE, "_build")
LIB = os.path.join(_VAR, "libsam3cu.so") if _VAR else os.path.join(HERE, "lib", "libsam3cu.so")
DEFS = os.environ.get("SAM3CU_BUILD_DEFS", "").split()
INC = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                  "-Xcompiler", "-fvisibility=hidden", "-I" + INC, "-I" + CSRC,
                  "--expt-relaxed-constexpr"]
CFLAGS = ["-O2", "-std=gnu11", "-fPIC", "-I" + INC, "-I" + CSRC]


def _newer(src_deps, obj):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in src_deps)


def _compile(src):
    base = os.path.splitext(os.path.basename(src))[0]
    obj = os.path.join(OBJ, base + ".o")
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INC, "*.h"))
    if not _newer([src] + headers + [__file__], obj):
        return obj, None
    if src.endswith(".cu"):
        cmd = [NVCC] + CUFLAGS + DEFS + ["-c", src, "-o", obj]
    else:
        cmd = ["gcc"] + CFLAGS + DEFS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    return obj, None


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.c")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(_compile, srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("libsam3cu build failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if _newer(objs, LIB):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print("linked", LIB)
    return LIB


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(OBJ, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    print(build(verbose=True))

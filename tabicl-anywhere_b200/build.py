"""Build the B200 backend's shared library (sm_100a) in-tree: tabicl-anywhere_b200/libtabicl_b200.so.

    python tabicl-anywhere_b200/build.py [--force]

nvcc cross-compiles for sm_100a without a GPU. The library links the CUDA runtime statically so it loads on
any machine with the driver, next to whatever runtime the host process (PyTorch, say) brings.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtabicl_b200.so")
SOURCES = ["kernels.cu", "attend_tc.cu", "gemm_tc.cu", "stage_rows.cu", "rows.cu", "qmlp_tc.cu", "tree.cu", "peer.cu", "fitcol.cu", "engine.cpp", "tier.cpp", "tirs.cpp", "noalloc.cu"]
HEADERS = ["device.cuh", "kernels.cuh", "tirs.hpp", "tc.cuh", "stage_common.cuh", "engine.hpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden,-ffp-contract=off",
    "-cudart", "static",
    "--expt-relaxed-constexpr",
]


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "tabicl_b200.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(p) > t for p in deps)


def build(force=False, verbose=False):
    if not force and not _stale():
        return LIB
    objs = []
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    # an object is rebuilt when it is older than its source, any header or this script
    newest_dep = max(os.path.getmtime(p) for p in [os.path.join(CSRC, h) for h in HEADERS] +
                     [os.path.join(HERE, "..", "include", "tabicl_b200.h"), os.path.abspath(__file__)])
    for src in SOURCES:
        obj = os.path.join(bdir, src + ".o")
        path = os.path.join(CSRC, src)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(newest_dep, os.path.getmtime(path)):
            cmd = [NVCC, *FLAGS, "-c", path, "-o", obj]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [NVCC, *FLAGS, "-shared", *objs, "-o", tmp]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

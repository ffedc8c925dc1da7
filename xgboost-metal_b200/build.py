"""Builds libxgboost.so (the CUDA trainer behind the upstream XGBoost C ABI)
for sm_100a, in-tree, into xgboost/lib/ next to the Python package.

Usage: python xgboost-metal_b200/build.py [--force]
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "xgboost", "lib")
LIB = os.path.join(LIB_DIR, "libxgboost.so")
ROOT = os.path.dirname(HERE)

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC",
          "-Xcompiler", "-ffp-contract=off", "-Xcompiler", "-fvisibility=hidden",
          "-I", CSRC, "-I", os.path.join(ROOT, "include")]
CUDA_ONLY = ["-Xptxas", "-O3", "--expt-relaxed-constexpr"]


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _compile(src):
    obj = os.path.join(BUILD, src + ".o")
    path = os.path.join(CSRC, src)
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    newest = max([os.path.getmtime(path)] + [os.path.getmtime(h) for h in headers])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    cmd = [NVCC] + ARCH + COMMON + (CUDA_ONLY if src.endswith(".cu") else ["-x", "cu"] + CUDA_ONLY)
    cmd += ["-c", path, "-o", obj]
    subprocess.run(cmd, check=True)
    return obj


def build(force=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(_compile, sources()))
    if os.path.exists(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-ldl"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))

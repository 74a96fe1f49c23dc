"""Build libzealot_rl.so in-tree with nvcc for sm_100a.

Usage: python -m zealot_b200.build [--force]

Every .cu/.cpp under zealot_b200/csrc is compiled for
``-gencode arch=compute_100a,code=sm_100a`` and linked with the static CUDA
runtime into ``zealot_b200/libzealot_rl.so``.  Host C++ is compiled with
``-ffp-contract=off`` so that f32 host arithmetic (the reference's Lcg and
initialisation) rounds like the Rust reference.
"""
from __future__ import annotations

import glob
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libzealot_rl.so")
OBJ = os.path.join(HERE, "_build")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr", "-Wno-deprecated-gpu-targets",
              f"-I{os.path.join(ROOT, 'include')}"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _fingerprint() -> str:
    h = hashlib.sha256()
    for f in _sources() + sorted(glob.glob(os.path.join(CSRC, "*.h")) +
                                 glob.glob(os.path.join(CSRC, "*.cuh"))) + \
            [os.path.join(ROOT, "include", "zealot_rl.h"), __file__]:
        with open(f, "rb") as fh:
            h.update(f.encode())
            h.update(fh.read())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> str:
    stamp = OUT + ".stamp"
    fp = _fingerprint()
    if not force and os.path.exists(OUT) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == fp:
                return OUT
    os.makedirs(OBJ, exist_ok=True)
    nvcc = _nvcc()

    def compile_one(src):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
        if src.endswith(".cpp"):
            cmd = [nvcc, "-x", "c++", *NVCC_FLAGS, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = OUT + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs,
           "-ldl", "-lpthread", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    with open(stamp, "w") as f:
        f.write(fp)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

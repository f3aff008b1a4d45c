"""Builds libigllm_cuda.so in-tree (igllm_b200/lib/) for sm_100a.

    python -m igllm_b200.build        # or: python igllm_b200/build.py

CUDA sources are compiled by nvcc with -gencode arch=compute_100a,code=sm_100a;
the host-C parts (n-gram scout, synthetic checkpoints) by gcc.  Objects go to
igllm_b200/_build/, the shared library to igllm_b200/lib/.
"""

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib")
TARGET = os.path.join(LIB, "libigllm_cuda.so")

CUDA_SOURCES = ["igc_kernels.cu", "igc_lanes.cu", "igc_runtime.cu", "igc_desk.cu"]
C_SOURCES = ["igc_synth.c", "igc_scout.c"]
HEADERS = ["igc_device.cuh", "igc_gemv.cuh", "igc_kernels.h", "igc_lanes.h", "igc_json.h", "igc_synth.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _newer(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.exists(s))


def build(verbose=False):
    """Compiles what changed and links libigllm_cuda.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    include = os.path.join(os.path.dirname(HERE), "include")
    deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(include, "igllm_cuda.h")]
    objects = []
    for src in CUDA_SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objects.append(obj)
        if _newer(obj, [path] + deps):
            cmd = [_nvcc()] + ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                                      "-c", path, "-o", obj]
            _run(cmd, verbose)
    for src in C_SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objects.append(obj)
        if _newer(obj, [path] + deps):
            _run(["gcc", "-std=c11", "-O2", "-fPIC", "-Wall", "-c", path, "-o", obj], verbose)
    if _newer(TARGET, objects):
        _run([_nvcc()] + ARCH + ["-shared", "-o", TARGET] + objects + ["-lpthread"], verbose)
    return TARGET


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError("build step failed: " + " ".join(cmd))


if __name__ == "__main__":
    print(build(verbose=True))

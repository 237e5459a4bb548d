"""Build recipe of libmomentum_compressor.so (sm_100a kernels + C host code).

Run ``python -m compressor_b200.build`` (or call ``build()``); the library is
written in-tree next to this file so it travels with the package.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libmomentum_compressor.so")
BUILD = os.path.join(HERE, "_build")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
CC = "/usr/bin/gcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

C_SOURCES = ["mc_util.c", "mc_wire.c", "mc_state.c", "mc_batch.c", "mc_api.c", "mc_replay.c", "mc_checkpoint.c"]
CU_SOURCES = ["mc_kernels.cu", "mc_noalloc.cu"]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]}")
    return r


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    inc = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-I" + os.path.join(CUDA, "include")]
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".h")]
    headers += [os.path.join(ROOT, "include", h) for h in os.listdir(os.path.join(ROOT, "include"))]
    objs = []
    for src in C_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if _stale(o, [s] + headers):
            _run([CC, "-std=gnu11", "-O2", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra",
                  "-Wno-unused-parameter", *inc, "-c", s, "-o", o])
        objs.append(o)
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        if _stale(o, [s] + headers) or ptxas_info:
            cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-fmad=false", "-std=c++17",
                   "-Xcompiler", "-fPIC,-fvisibility=hidden", *inc, "-c", s, "-o", o]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            r = _run(cmd)
            if ptxas_info or verbose:
                sys.stdout.write(r.stdout + r.stderr)
        objs.append(o)
    if _stale(OUT, objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", OUT, *objs,
              "-Xlinker", "--exclude-libs,ALL", "-ldl", "-lpthread", "-lrt"])
    return OUT


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="--ptxas" in sys.argv))

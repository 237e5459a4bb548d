"""Build recipe of the kernel-emulation library (test infrastructure only).

``build()`` compiles the library's C host code unchanged and its CUDA files
through the source transform in prep.py against emu.h and the fake runtime
in fake_cudart.cpp, into a shared library with the same C ABI as the product
library.  The CPU tests drive it exactly like the product library, so the
kernels' index arithmetic, bulk-copy alignment, shared-memory bounds, warp
exchanges and tile partitioning all run on the host against the oracle.  The
product library never contains any of this: without a GPU it fails loudly.

The output name carries a hash of every input, so an edited kernel is
always rebuilt.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
CSRC = os.path.join(ROOT, "compressor_b200", "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
C_SOURCES = ["mc_util.c", "mc_wire.c", "mc_state.c", "mc_batch.c", "mc_api.c", "mc_replay.c", "mc_checkpoint.c"]
# undefined-behaviour checks that need no preloaded runtime
SAN = ["-fsanitize=alignment,bounds,shift,signed-integer-overflow", "-fno-sanitize-recover=all"]


def _inputs():
    files = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))]
    files += [os.path.join(INCLUDE, f) for f in sorted(os.listdir(INCLUDE))]
    files += [os.path.join(HERE, f) for f in ("emu.h", "fake_cudart.cpp", "prep.py", "build.py")]
    return files


def _digest():
    h = hashlib.sha256()
    for f in _inputs():
        h.update(f.encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


def _run_all(cmds):
    procs = [(c, subprocess.Popen(c, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)) for c in cmds]
    for c, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            sys.stderr.write(" ".join(c) + "\n" + out)
            raise RuntimeError(f"emulator build step failed: {os.path.basename(c[-1])}")


def build() -> str:
    """Returns the path of the emulation library, building it if needed."""
    tag = _digest()
    out = os.path.join(BUILD, f"libmomentum_compressor_emu_{tag}.so")
    if os.path.exists(out):
        return out
    work = os.path.join(BUILD, tag)
    os.makedirs(work, exist_ok=True)
    sys.path.insert(0, HERE)
    try:
        import prep
    finally:
        sys.path.pop(0)
    kern = os.path.join(work, "emu_kernels.cpp")
    noalloc = os.path.join(work, "emu_noalloc.cpp")
    prep.main([os.path.join(CSRC, "mc_kernels.cu"), os.path.join(CSRC, "mc_noalloc.cu"), kern, noalloc])
    inc = ["-I" + HERE, "-I" + INCLUDE, "-I" + CSRC, "-I" + os.path.join(CUDA, "include")]
    common = ["-O1", "-g", "-fPIC", "-fvisibility=hidden", *SAN, *inc]
    cmds, objs = [], []
    for src in C_SOURCES:
        o = os.path.join(work, src + ".o")
        cmds.append(["gcc", "-std=gnu11", *common, "-c", os.path.join(CSRC, src), "-o", o])
        objs.append(o)
    for src in (kern, noalloc, os.path.join(HERE, "fake_cudart.cpp")):
        o = os.path.join(work, os.path.basename(src) + ".o")
        # -ffp-contract=off: no fused multiply-adds the kernels did not ask for
        cmds.append(["g++", "-std=c++17", "-ffp-contract=off", *common, "-c", src, "-o", o])
        objs.append(o)
    _run_all(cmds)
    tmp = out + ".tmp"
    _run_all([["g++", "-shared", *SAN, "-Wl,-Bsymbolic", "-Wl,--no-undefined", "-o", tmp, *objs,
               "-ldl", "-lpthread", "-lm"]])
    os.replace(tmp, out)
    for old in os.listdir(BUILD):   # builds of earlier sources
        if tag not in old:
            path = os.path.join(BUILD, old)
            shutil.rmtree(path) if os.path.isdir(path) else os.remove(path)
    return out


if __name__ == "__main__":
    print(build())

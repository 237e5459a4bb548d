"""Build recipe of the reference's own GPU code, used as a measured GPU
baseline beside this library (test and bench infrastructure; nothing in the
product loads it).

* ``v4``: the reference's fused q8 batch codec, a PyTorch extension
  (cuda_feasibility/falcom_cuda_v4/falcom_cuda_v4.cpp and
  falcom_cuda_v4_kernels.cu), compiled from its own sources with its own
  flags (cuda_feasibility/falcom_cuda_v4/setup.py:17-25) except the one arch
  flag: sm_70 there, sm_100a here.  Output: oracle/_ref/v4/_falcom_cuda_v4.so.
* ``microbench``: the reference's standalone six-kernel microbenchmark
  (cuda_feasibility/falcom_cuda_microbench.cu), compiled with nvcc -O3 for
  sm_100a.  Output: oracle/_ref/falcom_cuda_microbench.

The sources are read where they lie in the reference checkout
(oracle/reference_root.py); only the built files are kept, under
oracle/_ref/, which travels to the GPU box with the rest of the tree.

    python oracle/build_ref_gpu.py [v4] [microbench]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from oracle.reference_root import reference_root  # noqa: E402

OUT = os.path.join(HERE, "_ref")
V4_SO = os.path.join(OUT, "v4", "_falcom_cuda_v4.so")
MICROBENCH = os.path.join(OUT, "falcom_cuda_microbench")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def build_v4(ref: str) -> str:
    src = os.path.join(ref, "cuda_feasibility", "falcom_cuda_v4")
    from torch.utils.cpp_extension import load
    bdir = os.path.join(OUT, "v4_build")
    os.makedirs(bdir, exist_ok=True)
    load(name="_falcom_cuda_v4",
         sources=[os.path.join(src, "falcom_cuda_v4.cpp"), os.path.join(src, "falcom_cuda_v4_kernels.cu")],
         extra_cflags=["-O3", "-std=c++17"],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-std=c++17", ARCH],
         build_directory=bdir, verbose=False)
    os.makedirs(os.path.dirname(V4_SO), exist_ok=True)
    shutil.copy2(os.path.join(bdir, "_falcom_cuda_v4.so"), V4_SO)
    return V4_SO


def build_microbench(ref: str) -> str:
    src = os.path.join(ref, "cuda_feasibility", "falcom_cuda_microbench.cu")
    os.makedirs(OUT, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    subprocess.run([nvcc, "-O3", "-std=c++17", ARCH, src, "-o", MICROBENCH], check=True)
    return MICROBENCH


def main(argv) -> int:
    ref = reference_root()
    if not ref:
        print("reference checkout not found (FALCOM_REFERENCE_ROOT); nothing built")
        return 0
    what = argv or ["v4", "microbench"]
    if "microbench" in what:
        print(build_microbench(ref))
    if "v4" in what:
        print(build_v4(ref))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))

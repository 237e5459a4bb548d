"""Source transform of the library's CUDA files into host C++ for the kernel
emulator (emu.h).  Test infrastructure: the product library is built from the
untransformed sources by compressor_b200/build.py.

Kernel code stays as written; only the device-specific parts change:
qualifiers are dropped, __shared__ variables become static storage (one CTA
runs at a time), the inline-PTX helpers (bulk copies, mbarriers, L2 policies,
PDL) are replaced by host bodies that check what the hardware requires
(16-byte alignment, copies inside the CTA's dynamic shared memory), and each
launch runs its CTAs through emu_run().
"""
from __future__ import annotations

import re


def _replace_body(s: str, name: str, body: str) -> str:
    m = re.search(r"\n(inline )?[\w:<>\s\*]*\b" + name + r"\([^)]*\)\s*\{", s)
    if not m:
        raise ValueError(f"helper {name} not found in the kernel source")
    return _replace_block(s, s.index("{", m.start()), body)


def _replace_block(s: str, open_brace: int, body: str) -> str:
    depth, i = 0, open_brace
    while True:
        if s[i] == "{":
            depth += 1
        elif s[i] == "}":
            depth -= 1
            if depth == 0:
                break
        i += 1
    return s[: open_brace + 1] + body + s[i:]


HELPERS = {
    "pdl_wait": "",
    "pdl_release": "",
    "smem_u32": "return emu_smem_u32(p);",
    "mbar_init": "(void)bar; (void)count;",
    "mbar_expect_tx": "(void)bar; (void)bytes;",
    "l2_stream": "return 0;",
    "bulk_g2s": r"""
    (void)bar; (void)pol;
    char *d = (char *)emu_smem_ptr(dst);
    if ((dst & 15) || (((uintptr_t)src) & 15) || (bytes & 15)) {
        fprintf(stderr, "emu: bulk copy not 16-byte aligned (dst %u src %p bytes %u)\n", dst, src, bytes);
        abort();
    }
    if (d < (char *)emu_cta->lo || d + bytes > (char *)emu_cta->hi) {
        fprintf(stderr, "emu: bulk copy outside dynamic shared memory (dst %u bytes %u)\n", dst, bytes);
        abort();
    }
    memcpy(d, src, bytes);
""",
    "st_f4": r"""
    (void)pol;
    if (((uintptr_t)p) & 15) {
        fprintf(stderr, "emu: 16-byte store misaligned %p\n", (void *)p);
        abort();
    }
    *p = v;
""",
    # bulk copies complete at issue, so every phase a tile waits for is done
    "mbar_try_wait": "(void)bar; (void)parity; return true;",
    "mbar_wait": "(void)bar; (void)parity; return true;",
    # peer flags: kernels run one after another here, so a flag that is not
    # set yet never will be (one rank, or flags set beforehand)
    "st_release_sys": "__atomic_store_n(p, v, __ATOMIC_RELEASE);",
    "ld_acquire_sys": "return __atomic_load_n(p, __ATOMIC_ACQUIRE);",
    "wait_flags": r"""
    for (int k = 0; k < n; k++)
        if ((int32_t)(__atomic_load_n(p + k, __ATOMIC_ACQUIRE) - epoch) < 0) return false;
    return true;
""",
}

LAUNCH = re.compile(r"(\w+)<<<([^,]+),\s*(\w+),\s*([^,]+),\s*(\w+)>>>\((.*)\);")


def transform(src: str, helpers: bool) -> str:
    s = src.replace("#include <cuda_runtime.h>", '#include "emu.h"')
    s = re.sub(r"extern __shared__ __align__\(\d+\) float s_stage\[\];", "", s)
    s = re.sub(r"__launch_bounds__\([^)]*\)", "", s)
    s = s.replace("__device__ __forceinline__", "inline").replace("__forceinline__", "inline")
    s = s.replace("__global__", "").replace("__device__", "")
    s = re.sub(r"__align__\((\d+)\)", r"__attribute__((aligned(\1)))", s)
    s = s.replace("__shared__", "static")
    if helpers:
        for name, body in HELPERS.items():
            s = _replace_body(s, name, body)
    s = LAUNCH.sub(lambda m: (f"static_assert(({m.group(3)}) == EMU_TPB, \"block size\"); (void)({m.group(5)}); "
                              f"emu_run({m.group(2)}, {m.group(4)}, [&] {{ {m.group(1)}({m.group(6)}); }});"), s)
    m = re.search(r"static void launch_pdl\(void \(\*kern\)\(P\.\.\.\), int grid, size_t smem, "
                  r"cudaStream_t s, A\.\.\. args\) \{", s)
    if m:
        s = _replace_block(s, m.end() - 1, " (void)s; emu_run(grid, smem, [&] { kern(args...); }); ")
    return s


def main(argv):
    kernels, noalloc, out_kernels, out_noalloc = argv
    with open(kernels) as f:
        k = transform(f.read(), helpers=True)
    if "launch_pdl" in k and "emu_run(grid, smem" not in k:
        raise ValueError("launch_pdl not rewritten")
    with open(out_kernels, "w") as f:
        f.write(k)
    with open(noalloc) as f:
        n = transform(f.read(), helpers=False)
    if "<<<" in n or "<<<" in k:
        raise ValueError("a launch was not rewritten")
    with open(out_noalloc, "w") as f:
        f.write(n)


if __name__ == "__main__":
    import sys
    main(sys.argv[1:])

"""The struct layouts of include/momentum_compressor.h (compiled by gcc) equal
the ctypes mirror (compressor_b200/abi.py), which in turn mirrors the field
order that EB-FaLCom's FalComC.py binds (FalComC.py:47-105)."""
import ctypes
import os
import subprocess
import tempfile

from compressor_b200 import abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

STRUCTS = {
    "NDArray": abi.NDArrayC,
    "CompressorConfig": abi.CompressorConfigC,
    "CompressedLayerData": abi.CompressedLayerDataC,
    "BatchItem": abi.BatchItemC,
    "CompressionStats": abi.CompressionStatsC,
    "ClientStats": abi.ClientStatsC,
    "DetailedStats": abi.DetailedStatsC,
}


def test_layouts_match_header():
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "momentum_compressor.h"',
             "int main(void) {"]
    for cname, py in STRUCTS.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["/usr/bin/gcc", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    got = {}
    for line in out.splitlines():
        s, f, v = line.split()
        got[(s, f)] = int(v)
    for cname, py in STRUCTS.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def test_falcomc_field_order():
    """Field names and order bound by FalComC.py:47-105."""
    assert [f for f, _ in abi.NDArrayC._fields_] == ["data", "shape", "ndim", "total_size", "dtype"]
    assert [f for f, _ in abi.CompressorConfigC._fields_] == [
        "momentum_lr", "consistency_threshold", "lossless_compressor", "error_bounding_mode",
        "error_bound", "sz3_lib_path", "param_count_threshold", "max_history_length"]
    names = [f for f, _ in abi.CompressedLayerDataC._fields_]
    assert names[:12] == ["type", "codec", "data", "data_size", "bitmap", "bitmap_size",
                          "dominant_signs", "dominant_signs_size", "shape", "ndim",
                          "original_dtype", "stored_dtype"]
    assert names[-1] == "breakdown_total_time" and len(names) == 30

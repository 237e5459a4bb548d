"""CPU checks of the drop-in boundary: the library loads without a GPU and
exports every entry point declared in include/*.h."""
import ctypes
import os
import re

from compressor_b200.abi import ABI_SYMBOLS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b([a-z_][a-z0-9_]*)\s*\(", text):
            name = m.group(1)
            if name in ("defined", "sizeof", "if", "return"):
                continue
            # only declarations at statement level: "<type> [*]name("
            line_start = text.rfind("\n", 0, m.start()) + 1
            prefix = text[line_start:m.start()]
            if re.search(r"(void|int|char|NDArray|CompressedLayerData|MomentumCompressor|"
                         r"CompressionStats|DetailedStats|CompressorConfig|uint8_t|long long|"
                         r"falcom_replay|BatchItem|size_t|uint32_t)\s*\**\s*$", prefix):
                names.add(name)
    return names


def test_library_loads_and_exports_declared_symbols(product_lib):
    lib = ctypes.CDLL(product_lib)
    decl = declared_functions()
    assert len(decl) >= 45, sorted(decl)
    missing = [n for n in sorted(decl) if not hasattr(lib, n)]
    assert not missing, missing


def test_reference_abi_symbols_all_exported(product_lib):
    lib = ctypes.CDLL(product_lib)
    missing = [n for n in ABI_SYMBOLS if not hasattr(lib, n)]
    assert not missing, missing


def test_create_without_gpu_fails_loudly(product_lib):
    """No CUDA device in this container: create must refuse (NULL), never fall
    back to a host implementation."""
    try:
        import torch
        if torch.cuda.is_available():
            import pytest
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    from compressor_b200.abi import _bind
    lib = ctypes.CDLL(product_lib)
    _bind(lib)
    cfg = lib.momentum_compressor_default_config()
    assert abs(cfg.momentum_lr - 0.07) < 1e-7 and cfg.param_count_threshold == 1024
    assert not lib.momentum_compressor_create(ctypes.byref(cfg))


def test_host_only_helpers_without_gpu(product_lib):
    """ndarray_* helpers are plain host memory, as in the reference."""
    from compressor_b200.abi import _bind, NDArrayC
    lib = ctypes.CDLL(product_lib)
    _bind(lib)
    shape = (ctypes.c_size_t * 2)(3, 4)
    a = lib.ndarray_create(shape, 2, 0)
    assert a and a.contents.total_size == 12
    b = lib.ndarray_copy(a)
    assert b and b.contents.total_size == 12
    lib.ndarray_destroy(a)
    lib.ndarray_destroy(b)
    assert not lib.ndarray_create(shape, 0, 0)
    bad = (ctypes.c_size_t * 1)(0)
    assert not lib.ndarray_create(bad, 1, 0)

"""The codec's CUDA kernels, run on the CPU through the kernel emulator, against
the oracle.

tests/emu/build.py compiles mc_kernels.cu and mc_noalloc.cu through a source
transform into host C++ (one CTA at a time, its 256 threads on host threads,
warp shuffles and ballots emulated, bulk copies checked for 16-byte alignment
and for staying inside the CTA's dynamic shared memory, undefined-behaviour
checks on alignment, bounds, shifts and overflow), links them with the
unchanged host code and a fake CUDA runtime, and exposes the same C ABI as
the product library.  These tests drive that library exactly as the GPU
tests drive the product library, so a change to the kernels' indexing, tile
partitioning or codec arithmetic is checked here before it reaches a GPU.
Nothing here runs on, or stands in for, the GPU path: the product library
has no CPU fallback.
"""
import numpy as np
import pytest

from compressor_b200.abi import Codec
from oracle import binding as ob
from tests.helpers import decode_codes
from tests.parity_cases import check_encoder_decoder


@pytest.fixture(scope="module")
def emu_lib():
    from tests.emu import build as emu_build
    return emu_build.build()


@pytest.mark.parametrize("codec", ["raw", "q8", "int4"])
def test_emulated_kernels_match_oracle(emu_lib, codec):
    check_encoder_decoder(emu_lib, codec, n_rounds=4)


@pytest.mark.parametrize("codec", ["q8_raw", "int4_raw"])
def test_emulated_raw_payload_codecs(emu_lib, codec):
    # the codecs that store dequantised floats take the same quantiser path
    check_encoder_decoder(emu_lib, codec, n_rounds=3, seed=7)


def _noalloc_fn(path):
    import ctypes
    f = ctypes.CDLL(path).falcom_quantize_residual_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _oracle_payload(x, bits):
    scale, codes = ob.quantize(x, 127 if bits == 8 else 7)
    body = codes.tobytes() if bits == 8 else ob.pack_int4(codes).tobytes()
    return np.float32(scale).tobytes() + body


@pytest.mark.parametrize("bits", [8, 4])
def test_emulated_noalloc_quantiser(emu_lib, bits):
    """falcom_quantize_residual_noalloc: multi-tile and ragged sizes, 16-byte
    aligned input (vector path) and an input one float off (scalar path), two
    calls in a row on the same scratch, and an all-zero residual (scale 1)."""
    f = _noalloc_fn(emu_lib)
    assert f(None, 0, bits, None, None) == 0   # set-up only
    for n, off, seed in [(3 * 8192 + 5, 0, 1), (40_001, 1, 2), (8192, 0, 3), (7, 1, 4)]:
        x = np.zeros(n + 4, np.float32)
        x[off:off + n] = np.random.default_rng(seed).standard_normal(n).astype(np.float32) * (1 + seed)
        m = 4 + (n if bits == 8 else (n + 1) // 2)
        out = np.full(m + 8, 0xAB, np.uint8)
        assert f(x.ctypes.data + 4 * off, n, bits, out.ctypes.data, None) == 0
        assert out[:m].tobytes() == _oracle_payload(x[off:off + n], bits), (n, off)
        assert not np.any(out[m:] != 0xAB)   # nothing written past the payload
    z = np.zeros(1000, np.float32)
    out = np.empty(4 + 1000, np.uint8)
    assert f(z.ctypes.data, z.size, 8, out.ctypes.data, None) == 0
    assert np.frombuffer(out[:4].tobytes(), np.float32)[0] == 1.0 and not np.any(out[4:])


def test_emulated_noalloc_matches_batch_payload(emu_lib):
    """Same bytes as the batch entry point's payload for a fresh lossy tensor."""
    f = _noalloc_fn(emu_lib)
    x = np.random.default_rng(5).standard_normal(50_000).astype(np.float32)
    c = Codec(emu_lib, client="noalloc")
    assert c.lib.falcom_set_residual_codec(c.h, b"q8") == 0
    ret, layers, errs = c.compress_batch(["blocks.0.proj.weight"], [x])
    assert ret == 0, errs
    out = np.empty(4 + x.size, np.uint8)
    assert f(x.ctypes.data, x.size, 8, out.ctypes.data, None) == 0
    assert out.tobytes() == layers[0].data
    scale, codes = decode_codes(layers[0], x.size)
    es, ec = ob.quantize(x, 127)
    assert scale == es and np.array_equal(codes, ec)
    c.close()

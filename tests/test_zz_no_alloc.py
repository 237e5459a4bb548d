"""GPU test of falcom_quantize_residual_noalloc, the quantiser that uses a
fixed __device__ scratch array instead of allocating, for callers that cannot
allocate device memory (a framework's caching allocator owns it, or a
latency-critical path cannot afford cudaMalloc / cudaFree).  Its output must
equal the data payload that momentum_compressor_compress_batch writes for the
same tensor (a lossy float32 tensor with no history is quantised directly)
and the oracle's quantisation of the tensor, on two calls in a row, so the
scratch left by one call serves the next; and the device's free memory must
not change across calls.

The file name sorts last so it also runs after every other GPU test in one
process; it passes alone too."""
import ctypes

import numpy as np
import pytest

from compressor_b200.abi import Codec
from oracle import binding as ob
from tests.helpers import seeded

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

MAX_ELEMS = 8192 * 16384


def _lib(path):
    lib = ctypes.CDLL(path)
    f = lib.falcom_quantize_residual_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return lib


def _reference_payload(path, x, codec):
    """data payload of the batch entry point for a fresh lossy tensor."""
    c = Codec(path, client="noalloc")
    assert c.lib.falcom_set_residual_codec(c.h, codec.encode()) == 0
    ret, layers, errs = c.compress_batch(["blocks.0.proj.weight"], [x])
    assert ret == 0, errs
    L = layers[0]
    assert L.codec == codec, L.codec
    c.close()
    return L.data


def _noalloc(lib, x_dev, n, bits, out_dev, stream):
    return lib.falcom_quantize_residual_noalloc(ctypes.c_void_p(x_dev), n, bits, ctypes.c_void_p(out_dev),
                                                ctypes.c_void_p(stream))


def _payload_len(n, bits):
    return 4 + (n if bits == 8 else (n + 1) // 2)


def _check(got: bytes, want: bytes, bits: int):
    """Scale bit-identical; codes within one quantisation step (the tolerance
    of the codec's parity tests), and in practice identical."""
    assert len(got) == len(want)
    assert got[:4] == want[:4]
    if bits == 8:
        a = np.frombuffer(got[4:], np.int8).astype(np.int32)
        b = np.frombuffer(want[4:], np.int8).astype(np.int32)
    else:
        g, w = np.frombuffer(got[4:], np.uint8), np.frombuffer(want[4:], np.uint8)
        a = np.stack([g & 15, g >> 4], 1).reshape(-1).astype(np.int32)
        b = np.stack([w & 15, w >> 4], 1).reshape(-1).astype(np.int32)
    assert np.max(np.abs(a - b), initial=0) <= 1
    assert np.array_equal(a, b)


@pytest.mark.parametrize("bits,codec", [(8, "q8"), (4, "int4")])
@pytest.mark.parametrize("n", [1_000_003, 3 * 8192 + 5, 2_500_000])
def test_noalloc_matches_batch_payload_twice(product_lib, bits, codec, n):
    lib = _lib(product_lib)
    stream = torch.cuda.Stream()
    assert _noalloc(lib, 0, 0, bits, 0, stream.cuda_stream) == 0     # set-up only
    xs = [seeded((n,), 7 * n + k) * (1.0 + k) for k in range(2)]
    want = [_reference_payload(product_lib, x, codec) for x in xs]
    m = _payload_len(n, bits)
    # inputs and outputs are the test's own device buffers; the call itself allocates nothing
    outs = [torch.full((m,), 0xAB, dtype=torch.uint8, device="cuda") for _ in xs]
    xd = [torch.from_numpy(x).cuda() for x in xs]
    torch.cuda.synchronize()
    for x, o in zip(xd, outs):   # two calls in a row on one stream
        assert _noalloc(lib, x.data_ptr(), n, bits, o.data_ptr(), stream.cuda_stream) == 0
    stream.synchronize()
    for o, w, x in zip(outs, want, xs):
        got = o.cpu().numpy().tobytes()
        _check(got, w, bits)
        # and directly against the oracle's quantiser (scale bit-exact, codes equal)
        es, ec = ob.quantize(x, 127 if bits == 8 else 7)
        assert np.frombuffer(got[:4], np.float32)[0] == es
        codes = (np.frombuffer(got[4:], np.int8) if bits == 8
                 else ob.unpack_int4(np.frombuffer(got[4:], np.uint8), n))
        assert np.array_equal(codes.astype(np.int32), ec.astype(np.int32))


def test_noalloc_device_memory_unchanged(product_lib):
    """After a first call (set-up and the module's lazy loading), further
    calls leave the device's free memory exactly as it was: the entry point
    allocates nothing."""
    lib = _lib(product_lib)
    n = 2_000_000
    x = torch.from_numpy(seeded((n,), 5)).cuda()
    o = torch.empty(_payload_len(n, 8), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert _noalloc(lib, x.data_ptr(), n, 8, o.data_ptr(), s) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for bits in (8, 4, 8):
        assert _noalloc(lib, x.data_ptr(), n, bits, o.data_ptr(), s) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_unaligned_buffers_and_zero_residual(product_lib):
    """Odd input / output addresses take the scalar path; an all-zero residual
    gets scale 1 and zero codes, as in the batch entry point."""
    lib = _lib(product_lib)
    n = 70_001
    x = seeded((n,), 11)
    want = _reference_payload(product_lib, x, "q8")
    xbuf = torch.zeros(n + 1, dtype=torch.float32, device="cuda")
    xbuf[1:] = torch.from_numpy(x).cuda()
    obuf = torch.zeros(_payload_len(n, 8) + 3, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    s = torch.cuda.current_stream().cuda_stream
    assert _noalloc(lib, xbuf.data_ptr() + 4, n, 8, obuf.data_ptr() + 3, s) == 0
    torch.cuda.synchronize()
    _check(obuf.cpu().numpy().tobytes()[3:], want, 8)
    z = torch.zeros(n, dtype=torch.float32, device="cuda")
    o2 = torch.empty(_payload_len(n, 8), dtype=torch.uint8, device="cuda")
    assert _noalloc(lib, z.data_ptr(), n, 8, o2.data_ptr(), s) == 0
    torch.cuda.synchronize()
    got = o2.cpu().numpy().tobytes()
    assert np.frombuffer(got[:4], np.float32)[0] == 1.0 and not any(got[4:])
    assert got == _reference_payload(product_lib, np.zeros(n, np.float32), "q8")


def test_noalloc_rejects_sizes_beyond_scratch(product_lib):
    """n above the scratch bound, and bad arguments, are refused before any
    launch; a valid call afterwards still works."""
    lib = _lib(product_lib)
    x = torch.ones(16, dtype=torch.float32, device="cuda")
    o = torch.zeros(20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert _noalloc(lib, x.data_ptr(), MAX_ELEMS + 1, 8, o.data_ptr(), s) == -4
    assert _noalloc(lib, x.data_ptr(), 16, 5, o.data_ptr(), s) == -4
    assert _noalloc(lib, 0, 16, 8, o.data_ptr(), s) == -4
    assert _noalloc(lib, x.data_ptr(), 16, 8, o.data_ptr(), s) == 0
    torch.cuda.synchronize()
    got = o.cpu().numpy().tobytes()
    assert np.frombuffer(got[:4], np.float32)[0] == np.float32(1.0) / np.float32(127.0)
    assert np.array_equal(np.frombuffer(got[4:], np.int8), np.full(16, 127, np.int8))

"""GPU tests of the memory-residency and framing paths of the codec: device
vs host buffers, in-place vs expanded frame reads, aligned (float4) vs
unaligned element access, foreign zstd frames.  Every path must produce the
same bytes as the host path, which test_gpu_parity checks against the oracle."""
import ctypes

import numpy as np
import pytest

from compressor_b200.abi import Codec, DeviceArray, HostArray, Layer, ndarray_to_numpy
from oracle import binding as ob
from tests.helpers import seeded

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SHAPES = [("a.weight", (96, 64, 3, 3)), ("b.weight", (256, 128, 1, 1)), ("c.weight", (33, 7, 2, 2)),
          ("d.bias", (100,)), ("e.weight", (10, 300))]


def make(seed):
    return [seeded(s, seed * 10 + i) for i, (_, s) in enumerate(SHAPES)]


def host_args(xs):
    hs = [HostArray(x) for x in xs]
    return hs, hs


def device_args(offset_elems=0):
    def f(xs):
        ts, arrs = [], []
        for x in xs:
            t = torch.zeros(x.size + offset_elems, dtype=torch.float32, device="cuda")
            t[offset_elems:] = torch.from_numpy(x.reshape(-1)).cuda()
            ts.append(t)
            arrs.append(DeviceArray(t.data_ptr() + 4 * offset_elems, x.shape))
        torch.cuda.synchronize()
        return arrs, ts
    return f


def closed_loop(lib, rounds, to_args, codec="q8"):
    """Returns per round: payload bytes of every layer and decoded outputs."""
    enc = Codec(lib, client="c0", param_count_threshold=16)
    dec = Codec(lib, client="c0", param_count_threshold=16)
    enc.lib.falcom_set_residual_codec(enc.h, codec.encode())
    names = [n for n, _ in SHAPES]
    from compressor_b200.abi import NDArrayC
    out = []
    for xs in rounds:
        args, keep = to_args(xs)
        ret, items = enc.compress_batch_raw(names, args)
        assert ret == 0, enc.lib.falcom_last_error(enc.h)
        payload = []
        for it in items:
            c = it.compressed.contents
            blobs = []
            for ptr, size in ((c.data, c.data_size), (c.bitmap, c.bitmap_size),
                              (c.dominant_signs, c.dominant_signs_size)):
                if not ptr or size == 0:
                    blobs.append(b"")
                    continue
                addr = ctypes.cast(ptr, ctypes.c_void_p).value
                if enc.lib.falcom_is_device_pointer(ctypes.c_void_p(addr)):
                    t = torch.empty(size, dtype=torch.uint8, device="cuda")
                    torch.cuda.synchronize()
                    cudart_copy(t.data_ptr(), addr, size)
                    blobs.append(t.cpu().numpy().tobytes())
                else:
                    blobs.append(ctypes.string_at(addr, size))
            payload.append(tuple(blobs))
        n = len(names)
        outs = (ctypes.POINTER(NDArrayC) * n)()
        r2 = dec.lib.momentum_compressor_decompress_batch(dec.h, items, n, b"c0", outs)
        assert r2 == 0, dec.lib.falcom_last_error(dec.h)
        decoded = []
        for i in range(n):
            a = outs[i].contents
            if dec.lib.falcom_is_device_pointer(ctypes.c_void_p(a.data)):
                t = torch.empty(a.total_size, dtype=torch.float32, device="cuda")
                torch.cuda.synchronize()
                cudart_copy(t.data_ptr(), a.data, a.total_size * 4)
                decoded.append(t.cpu().numpy())
            else:
                decoded.append(ndarray_to_numpy(outs[i]).reshape(-1))
            dec.lib.ndarray_destroy(outs[i])
        enc.free_items(items)
        out.append((payload, decoded))
    enc.close()
    dec.close()
    return out


def cudart_copy(dst, src, nbytes):
    """Device-to-device copy of raw addresses through torch."""
    class _Arr:
        def __init__(self, ptr):
            self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                             "version": 3, "strides": None}
    torch.as_tensor(_Arr(dst), device="cuda").copy_(torch.as_tensor(_Arr(src), device="cuda"))
    torch.cuda.synchronize()


def assert_same(a, b):
    for (pa, da), (pb, db) in zip(a, b):
        assert pa == pb
        for x, y in zip(da, db):
            assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("codec", ["q8", "int4", "raw"])
def test_device_inputs_match_host_inputs(product_lib, codec):
    rounds = [make(s) for s in range(3)]
    h = closed_loop(product_lib, rounds, host_args, codec)
    d = closed_loop(product_lib, rounds, device_args(0), codec)
    assert_same(h, d)


def test_unaligned_device_inputs_take_scalar_path(product_lib):
    rounds = [make(s) for s in range(3)]
    h = closed_loop(product_lib, rounds, host_args)
    d = closed_loop(product_lib, rounds, device_args(1))   # 4-byte offset: no float4 access
    assert_same(h, d)


def _struct_at(layer, blobs_at):
    """CompressedLayerDataC whose payload pointers are the given addresses."""
    c, _ = Layer(**{**layer.__dict__, "data": b"", "bitmap": b"", "dominant_signs": b""}).to_c()
    for name, (addr, size) in blobs_at.items():
        setattr(c, name, ctypes.cast(ctypes.c_void_p(addr), ctypes.POINTER(ctypes.c_uint8)) if addr else None)
        setattr(c, name + "_size", size)
    return c


def _decode_structs(codec, names, structs):
    from compressor_b200.abi import BatchItemC, NDArrayC
    n = len(names)
    items = (BatchItemC * n)()
    enc = [nm.encode() for nm in names]
    for i in range(n):
        items[i].layer_name = enc[i]
        items[i].compressed = ctypes.pointer(structs[i])
    outs = (ctypes.POINTER(NDArrayC) * n)()
    ret = codec.lib.momentum_compressor_decompress_batch(codec.h, items, n, b"c0", outs)
    res = []
    for i in range(n):
        if not outs[i]:
            res.append(None)
            continue
        a = outs[i].contents
        if codec.lib.falcom_is_device_pointer(ctypes.c_void_p(a.data)):
            t = torch.empty(a.total_size, dtype=torch.float32, device="cuda")
            cudart_copy(t.data_ptr(), a.data, a.total_size * 4)
            res.append(t.cpu().numpy())
        else:
            res.append(ndarray_to_numpy(outs[i]).reshape(-1))
        codec.lib.ndarray_destroy(outs[i])
    return ret, res


def test_foreign_frames_are_expanded(product_lib):
    """Payloads at odd host addresses, and payloads copied into device memory
    the library does not own, decode exactly like the library's own."""
    enc = Codec(product_lib, client="c0", param_count_threshold=16)
    dec_ref = Codec(product_lib, client="c0", param_count_threshold=16)
    dec_odd = Codec(product_lib, client="c0", param_count_threshold=16)
    dec_dev = Codec(product_lib, client="c0", param_count_threshold=16)
    names = [n for n, _ in SHAPES]
    for s in range(3):
        ret, layers, _ = enc.compress_batch(names, make(s))
        assert ret == 0
        r0, y0 = dec_ref.decompress_batch(names, layers)
        assert r0 == 0
        # odd host addresses
        total = sum(len(L.data) + len(L.bitmap) + len(L.dominant_signs) + 3 for L in layers) + 16
        host = (ctypes.c_uint8 * total)()
        base = ctypes.addressof(host)
        off = 1
        odd_structs = []
        dev_structs = []
        dev_keep = []
        for L in layers:
            at = {}
            dat = {}
            for name in ("data", "bitmap", "dominant_signs"):
                blob = getattr(L, name)
                if not blob:
                    at[name] = (0, 0)
                    dat[name] = (0, 0)
                    continue
                ctypes.memmove(base + off, blob, len(blob))
                at[name] = (base + off, len(blob))
                off += len(blob) + 1
                t = torch.tensor(np.frombuffer(blob, np.uint8), device="cuda")
                dev_keep.append(t)
                dat[name] = (t.data_ptr(), len(blob))
            odd_structs.append(_struct_at(L, at))
            dev_structs.append(_struct_at(L, dat))
        torch.cuda.synchronize()
        r1, y1 = _decode_structs(dec_odd, names, odd_structs)
        r2, y2 = _decode_structs(dec_dev, names, dev_structs)
        assert r1 == 0 and r2 == 0
        for a, b, c in zip(y0, y1, y2):
            a = a.reshape(-1)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
            assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


def test_reference_frames_with_compressed_blocks(product_lib):
    """libzstd level-10 frames (compressed blocks) are decoded through the
    host libzstd path and give the same result as GPU-written frames."""
    a = Codec(product_lib, client="c0", param_count_threshold=16)
    b = Codec(product_lib, client="c0", param_count_threshold=16)
    assert b.lib.falcom_set_frame_mode(b.h, b"libzstd") == 0
    da = Codec(product_lib, client="c0", param_count_threshold=16)
    db = Codec(product_lib, client="c0", param_count_threshold=16)
    names = [n for n, _ in SHAPES]
    for s in range(3):
        xs = make(s)
        _, LA, _ = a.compress_batch(names, xs)
        _, LB, _ = b.compress_batch(names, xs)
        for la, lb in zip(LA, LB):
            assert ob.zstd_decompress(la.bitmap) == ob.zstd_decompress(lb.bitmap) if la.bitmap else True
        _, ya = da.decompress_batch(names, LA)
        _, yb = db.decompress_batch(names, LB)
        for x, y in zip(ya, yb):
            assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


def test_copy_sm_pinned_host_and_device(product_lib):
    """falcom_copy_sm between torch's pinned host memory and device memory in
    both directions: sizes with ragged heads and tails, congruent and
    incongruent offsets, device to device; bytes outside the range untouched;
    pageable host memory refused."""
    lib = ctypes.CDLL(product_lib)
    lib.falcom_copy_sm.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    lib.falcom_copy_sm.restype = ctypes.c_int
    cap = 1 << 22
    g = torch.Generator().manual_seed(7)
    h = torch.randint(0, 256, (cap,), dtype=torch.uint8, generator=g).pin_memory()
    d = torch.randint(0, 256, (cap,), dtype=torch.uint8, generator=g).cuda()
    d2 = torch.zeros(cap, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for n, so, do in ((0, 0, 0), (1, 0, 0), (15, 1, 1), (17, 3, 3), (1000, 5, 9), (3_000_001, 16, 48),
                      (3_000_000, 7, 7), (1 << 21, 0, 0)):
        for src, dst in ((h, d), (d, h), (d, d2)):
            before = dst.cpu().clone()
            assert lib.falcom_copy_sm(dst.data_ptr() + do, src.data_ptr() + so, n, 0, s) == 0
            torch.cuda.synchronize()
            got = dst.cpu()
            assert torch.equal(got[do:do + n], src.cpu()[so:so + n]), (n, so, do)
            assert torch.equal(got[:do], before[:do]) and torch.equal(got[do + n:], before[do + n:])
    pageable = torch.zeros(64, dtype=torch.uint8)
    assert lib.falcom_copy_sm(d.data_ptr(), pageable.data_ptr(), 64, 0, s) == -4

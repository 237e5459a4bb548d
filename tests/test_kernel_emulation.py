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


def test_emulated_aggregate_add_and_store(emu_lib):
    """Weighted aggregate fused into the decoder's reconstruct kernel: three
    clients added into a cleared buffer equal the host's fma chain bit for
    bit; the first client in store mode over a NaN-filled buffer gives the
    same bits, and so does a third server in aggregate-only mode (no decoded
    arrays for the float32 items, the int64 item still returned); the int64
    item is never added."""
    import ctypes
    lib = ctypes.CDLL(emu_lib)
    lib.emu_device_alloc.restype = ctypes.c_void_p
    lib.emu_device_alloc.argtypes = [ctypes.c_size_t]
    lib.emu_device_free.argtypes = [ctypes.c_void_p]
    shapes = [("l1.conv.weight", (16, 8, 3, 3)), ("l1.bn.bias", (16,)), ("l2.conv.weight", (32, 16, 1, 1)),
              ("fc.weight", (10, 64)), ("l1.bn.num_batches_tracked", (1,))]
    names = [n for n, _ in shapes]
    sizes = [int(np.prod(s)) for _, s in shapes]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(int)
    total = int(sum(sizes))
    off_c = (ctypes.c_size_t * len(names))(*[int(o) for o in offs])
    weights = [0.5, 0.3, 0.2]
    encs = [Codec(emu_lib, client=f"c{c}", param_count_threshold=16) for c in range(3)]
    add_srv = Codec(emu_lib, client="server", param_count_threshold=16)
    st_srv = Codec(emu_lib, client="server", param_count_threshold=16)
    ao_srv = Codec(emu_lib, client="server", param_count_threshold=16)
    pa, pb, pc = (lib.emu_device_alloc(4 * total) for _ in range(3))
    a = np.ctypeslib.as_array((ctypes.c_float * total).from_address(pa))
    b = np.ctypeslib.as_array((ctypes.c_float * total).from_address(pb))
    ao = np.ctypeslib.as_array((ctypes.c_float * total).from_address(pc))
    rng = np.random.default_rng(3)
    for t in range(2):
        a[:] = 0.0
        b[:] = np.nan
        ao[:] = np.nan
        want = np.zeros(total, np.float32)
        for c in range(3):
            xs = [np.array([t + 1], np.int64) if n.endswith("tracked") else
                  (rng.standard_normal(s) * 1e-3).astype(np.float32) for n, s in shapes]
            ret, layers, errs = encs[c].compress_batch(names, xs)
            assert ret == 0, errs
            for srv, p in ((add_srv, pa), (st_srv, pb), (ao_srv, pc)):
                assert srv.lib.falcom_set_aggregate(srv.h, ctypes.c_void_p(p), off_c, len(names), weights[c]) == 0
            for srv in (st_srv, ao_srv):
                assert srv.lib.falcom_set_aggregate_store(srv.h, 1 if c == 0 else 0) == 0
            assert ao_srv.lib.falcom_set_aggregate_only(ao_srv.h, 1) == 0
            ret, outs = add_srv.decompress_batch(names, layers, client=f"c{c}")
            assert ret == 0 and st_srv.decompress_batch(names, layers, client=f"c{c}")[0] == 0
            ret, ao_outs = ao_srv.decompress_batch(names, layers, client=f"c{c}")
            assert ret == 0
            for (n, _), o in zip(shapes, ao_outs):
                assert (o is not None) == n.endswith("tracked"), n
            for i, o in enumerate(outs):
                if o.dtype == np.float32:   # the kernel's fma chain, restated with exact float64 products
                    seg = want[offs[i]:offs[i] + sizes[i]]
                    seg[:] = (np.float64(np.float32(weights[c])) * o.reshape(-1) + seg).astype(np.float32)
        for i, (n, _) in enumerate(shapes):
            ra, rb, rc, rw = (v[offs[i]:offs[i] + sizes[i]] for v in (a, b, ao, want))
            if n.endswith("tracked"):
                assert not ra.any() and np.isnan(rb).all() and np.isnan(rc).all()
            else:
                assert np.array_equal(ra.view(np.uint32), rb.view(np.uint32)), n
                assert np.array_equal(ra.view(np.uint32), rc.view(np.uint32)), n
                assert np.array_equal(ra.view(np.uint32), rw.view(np.uint32)), n
    for c in encs + [add_srv, st_srv, ao_srv]:
        c.close()
    for p in (pa, pb, pc):
        lib.emu_device_free(p)


def test_emulated_sharded_aggregate_two_ranks(emu_lib):
    """The sharded aggregate (a reduce-scatter fused into the decoder, then
    the shard sum and all-gather kernel), with two ranks emulated in one
    process: rank 0 decodes clients A1 (into its local aggregate) and A2
    (added to it, the sum stored into the owners' landing slots), rank 1
    decodes client B (stored into the landing slots); then each rank's
    falcom_shard_reduce sums its shard and stores it into both aggregates.
    With power-of-two weights every product is exact, so both aggregates
    must equal (0.25 xA1 + 0.25 xA2) + 0.5 xB in float32 bit for bit, x the
    clients' decodes from a plain decoder; padding between items stays 0."""
    import ctypes
    lib = ctypes.CDLL(emu_lib)
    lib.emu_device_alloc.restype = ctypes.c_void_p
    lib.emu_device_alloc.argtypes = [ctypes.c_size_t]
    lib.emu_device_free.argtypes = [ctypes.c_void_p]
    shapes = [("l1.conv.weight", (32, 16, 3, 3)), ("l1.bn.bias", (32,)), ("l2.conv.weight", (64, 32, 1, 1)),
              ("fc.weight", (10, 300)), ("fc.bias", (10,))]
    names = [n for n, _ in shapes]
    sizes = [int(np.prod(s)) for _, s in shapes]
    offs, o = [], 0
    for n_ in sizes:
        offs.append(o)
        o = (o + n_ + 63) // 64 * 64
    total = o
    nranks, shard = 2, max(4096, ((total + 1) // 2 + 63) // 64 * 64)
    off_c = (ctypes.c_size_t * len(names))(*offs)
    c_vp = ctypes.c_void_p
    land = [lib.emu_device_alloc(4 * nranks * shard) for _ in range(nranks)]
    aggs = [lib.emu_device_alloc(4 * nranks * shard) for _ in range(nranks)]
    view = lambda p, n: np.ctypeslib.as_array((ctypes.c_float * n).from_address(p))
    for p in land + aggs:
        view(p, nranks * shard)[:] = 0.0
    land_arr = (c_vp * nranks)(*land)
    agg_arr = (c_vp * nranks)(*aggs)
    enc = {c: Codec(emu_lib, client=c, param_count_threshold=16) for c in ("A1", "A2", "B")}
    srv = [Codec(emu_lib, client="server", param_count_threshold=16) for _ in range(nranks)]
    plain = Codec(emu_lib, client="server", param_count_threshold=16)
    w = {"A1": 0.25, "A2": 0.25, "B": 0.5}
    rank_of = {"A1": 0, "A2": 0, "B": 1}
    rng = np.random.default_rng(11)
    for t in range(3):
        dec = {}
        for c in ("A1", "A2", "B"):
            xs = [(rng.standard_normal(s) * 1e-3).astype(np.float32) for _, s in shapes]
            ret, layers, errs = enc[c].compress_batch(names, xs)
            assert ret == 0, errs
            r = rank_of[c]
            sv = srv[r]
            assert sv.lib.falcom_set_aggregate(sv.h, c_vp(aggs[r]), off_c, len(names), w[c]) == 0
            assert sv.lib.falcom_set_aggregate_store(sv.h, 0 if c == "A2" else 1) == 0
            assert sv.lib.falcom_set_aggregate_only(sv.h, 1) == 0
            last = c in ("A2", "B")   # the rank's last client writes into the landing slots
            if last:
                assert sv.lib.falcom_set_aggregate_shards(sv.h, land_arr, nranks, r, shard) == 0
            else:
                assert sv.lib.falcom_set_aggregate_shards(sv.h, None, 0, 0, 0) == 0
            assert sv.decompress_batch(names, layers, client=c)[0] == 0
            ret, outs = plain.decompress_batch(names, layers, client=c)
            assert ret == 0
            dec[c] = outs
        for r in range(nranks):
            assert lib.falcom_shard_reduce(c_vp(land[r]), nranks, r, shard, total, agg_arr, None) == 0
        for i, n_ in enumerate(sizes):
            xa1, xa2, xb = (dec[c][i].reshape(-1) for c in ("A1", "A2", "B"))
            want = ((np.float32(0.25) * xa1) + (np.float32(0.25) * xa2)) + np.float32(0.5) * xb
            for r in range(nranks):
                got = view(aggs[r], total)[offs[i]:offs[i] + n_]
                assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32)), (t, r, names[i])
        for r in range(nranks):
            a = view(aggs[r], total).copy()
            mask = np.ones(total, bool)
            for i, n_ in enumerate(sizes):
                mask[offs[i]:offs[i] + n_] = False
            assert not a[mask].any()        # padding between items untouched
    # an item outside the shards is refused before any launch
    sv = srv[0]
    assert 2 * 4096 < total
    assert sv.lib.falcom_set_aggregate_shards(sv.h, land_arr, nranks, 0, 4096) == 0
    ret, layers, _ = enc["A1"].compress_batch(names, [(rng.standard_normal(s) * 1e-3).astype(np.float32)
                                                      for _, s in shapes])
    assert ret == 0
    assert sv.decompress_batch(names, layers, client="A1")[0] != 0
    assert sv.lib.falcom_set_aggregate_shards(sv.h, land_arr, nranks, 2, shard) == -4      # rank out of range
    assert sv.lib.falcom_set_aggregate_shards(sv.h, land_arr, nranks, 0, 100) == -4        # shard not a multiple of 64
    for c in list(enc.values()) + srv + [plain]:
        c.close()
    for p in land + aggs:
        lib.emu_device_free(p)


def test_emulated_peer_allreduce_in_place(emu_lib):
    """The one-shot in-place all-reduce (falcom_peer_allreduce) over three
    emulated ranks' aggregates, a total that is not a multiple of 4 (the
    last rank's range ends in a partial quad) and a rank whose range is
    empty: after every rank's call every aggregate holds (a0 + a1) + a2 in
    float32 bit for bit, elements past `total` untouched."""
    import ctypes
    lib = ctypes.CDLL(emu_lib)
    lib.emu_device_alloc.restype = ctypes.c_void_p
    lib.emu_device_alloc.argtypes = [ctypes.c_size_t]
    lib.emu_device_free.argtypes = [ctypes.c_void_p]
    lib.falcom_peer_allreduce.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                          ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]
    c_vp = ctypes.c_void_p
    view = lambda p, n: np.ctypeslib.as_array((ctypes.c_float * n).from_address(p))
    rng = np.random.default_rng(5)
    for nranks, shard, total in ((3, 4096, 2 * 4096 + 1234 + 3), (3, 8192, 8192 + 77), (2, 4096, 4096)):
        cap = nranks * shard
        aggs = [lib.emu_device_alloc(4 * cap) for _ in range(nranks)]
        init = [(rng.standard_normal(cap) * 1e-3).astype(np.float32) for _ in range(nranks)]
        for p, a in zip(aggs, init):
            view(p, cap)[:] = a
        arr = (c_vp * nranks)(*aggs)
        for r in range(nranks):
            assert lib.falcom_peer_allreduce(arr, nranks, r, shard, total, None) == 0
        want = init[0][:total].copy()
        for a in init[1:]:
            want = want + a[:total]
        for r in range(nranks):
            got = view(aggs[r], cap)
            assert np.array_equal(got[:total].view(np.uint32), want.view(np.uint32)), (nranks, shard, total, r)
            assert np.array_equal(got[total:].view(np.uint32), init[r][total:].view(np.uint32))
        for p in aggs:
            lib.emu_device_free(p)
    arr = (c_vp * 2)(None, None)
    assert lib.falcom_peer_allreduce(arr, 2, 0, 4096, 4096, None) == -4      # NULL aggregates
    assert lib.falcom_peer_allreduce(arr, 9, 0, 4096, 4096, None) == -4      # too many ranks


def test_emulated_copy_sm(emu_lib):
    """falcom_copy_sm (the SM copy kernel) between pinned host and device
    buffers of the emulator: every size from 0 to 70 bytes and a large one,
    congruent and incongruent offsets of source and destination, bytes
    outside the range untouched; pageable memory and NULL refused."""
    import ctypes
    lib = ctypes.CDLL(emu_lib)
    lib.emu_device_alloc.restype = ctypes.c_void_p
    lib.emu_device_alloc.argtypes = [ctypes.c_size_t]
    lib.emu_device_free.argtypes = [ctypes.c_void_p]
    lib.emu_host_alloc.restype = ctypes.c_void_p
    lib.emu_host_alloc.argtypes = [ctypes.c_size_t]
    lib.emu_host_free.argtypes = [ctypes.c_void_p]
    lib.falcom_copy_sm.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    cap = 1 << 16
    h = lib.emu_host_alloc(cap)
    d = lib.emu_device_alloc(cap)
    view = lambda p: np.ctypeslib.as_array((ctypes.c_uint8 * cap).from_address(p))
    rng = np.random.default_rng(3)
    cases = [(n, so, do) for n in range(0, 71) for so, do in ((0, 0), (3, 3), (5, 9))]
    cases += [(40000, 16, 48), (40000, 7, 7), (40001, 1, 2)]
    for n, so, do in cases:
        for src, dst in ((h, d), (d, h)):
            view(src)[:] = rng.integers(0, 256, cap, dtype=np.uint8)
            before = view(dst).copy()
            assert lib.falcom_copy_sm(dst + do, src + so, n, 3, None) == 0
            got = view(dst)
            assert np.array_equal(got[do:do + n], view(src)[so:so + n]), (n, so, do)
            assert np.array_equal(got[:do], before[:do]) and np.array_equal(got[do + n:], before[do + n:])
    pageable = (ctypes.c_uint8 * 64)()
    assert lib.falcom_copy_sm(d, ctypes.addressof(pageable), 64, 0, None) == -4
    assert lib.falcom_copy_sm(None, h, 64, 0, None) == -4
    assert lib.falcom_copy_sm(d, h, cap + 1, 0, None) == -4     # the source range ends outside the pinned buffer
    lib.emu_host_free(h)
    lib.emu_device_free(d)


@pytest.mark.parametrize("nranks", [8])
def test_emulated_sharded_aggregate_many_ranks(emu_lib, nranks):
    """The fused sharded aggregate and the one-shot all-reduce with 8
    emulated ranks (the most either supports), one client per rank, weight 1/nranks (a power of two, so
    every weighted decode is exact): after each rank's falcom_shard_reduce
    every aggregate equals the rank-order float32 sum of the weighted
    decodes bit for bit, and so does the one-shot all-reduce of plain local
    aggregates; ranks whose shards lie past the last element store nothing."""
    import ctypes
    lib = ctypes.CDLL(emu_lib)
    lib.emu_device_alloc.restype = ctypes.c_void_p
    lib.emu_device_alloc.argtypes = [ctypes.c_size_t]
    lib.emu_device_free.argtypes = [ctypes.c_void_p]
    lib.falcom_peer_allreduce.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                          ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]
    shapes = [("l1.conv.weight", (32, 16, 3, 3)), ("l1.bn.bias", (32,)), ("l2.conv.weight", (64, 32, 1, 1)),
              ("fc.weight", (10, 300)), ("fc.bias", (10,))]
    names = [n for n, _ in shapes]
    sizes = [int(np.prod(s)) for _, s in shapes]
    offs, o = [], 0
    for n_ in sizes:
        offs.append(o)
        o = (o + n_ + 63) // 64 * 64
    total = o
    shard = max(4096, ((total + nranks - 1) // nranks + 63) // 64 * 64)
    assert total <= (nranks - 1) * shard            # the last rank's shard is empty
    off_c = (ctypes.c_size_t * len(names))(*offs)
    c_vp = ctypes.c_void_p
    cap = nranks * shard
    land = [lib.emu_device_alloc(4 * cap) for _ in range(nranks)]
    aggs = [lib.emu_device_alloc(4 * cap) for _ in range(nranks)]
    plain = [lib.emu_device_alloc(4 * cap) for _ in range(nranks)]
    view = lambda p, n: np.ctypeslib.as_array((ctypes.c_float * n).from_address(p))
    for p in land + aggs + plain:
        view(p, cap)[:] = 0.0
    land_arr = (c_vp * nranks)(*land)
    agg_arr = (c_vp * nranks)(*aggs)
    plain_arr = (c_vp * nranks)(*plain)
    w = 1.0 / nranks
    rng = np.random.default_rng(21)
    mk = lambda cid: Codec(emu_lib, client=cid, param_count_threshold=16)
    encs = [mk(f"C{r}") for r in range(nranks)]
    srvs = [mk("server") for r in range(nranks)]
    refs = [mk("server") for r in range(nranks)]
    for t in range(3):   # round 0 direct, then momentum
        want = np.zeros(total, np.float32)
        for r in range(nranks):
            cid = f"C{r}"
            enc, srv, ref = encs[r], srvs[r], refs[r]
            xs = [(rng.standard_normal(s) * 1e-3).astype(np.float32) for _, s in shapes]
            ret, layers, errs = enc.compress_batch(names, xs)
            assert ret == 0, errs
            for sv, agg in ((srv, aggs[r]), (ref, plain[r])):
                assert sv.lib.falcom_set_aggregate(sv.h, c_vp(agg), off_c, len(names), w) == 0
                assert sv.lib.falcom_set_aggregate_store(sv.h, 1) == 0
                assert sv.lib.falcom_set_aggregate_only(sv.h, 1) == 0
            assert srv.lib.falcom_set_aggregate_shards(srv.h, land_arr, nranks, r, shard) == 0
            assert srv.decompress_batch(names, layers, client=cid)[0] == 0
            assert ref.decompress_batch(names, layers, client=cid)[0] == 0
            flat = view(plain[r], cap)[:total].copy()
            want = want + flat          # rank order
        for r in range(nranks):
            assert lib.falcom_shard_reduce(c_vp(land[r]), nranks, r, shard, total, agg_arr, None) == 0
        for r in range(nranks):
            assert lib.falcom_peer_allreduce(plain_arr, nranks, r, shard, total, None) == 0
        for r in range(nranks):
            assert np.array_equal(view(aggs[r], cap)[:total].view(np.uint32), want.view(np.uint32)), (t, r)
            assert np.array_equal(view(plain[r], cap)[:total].view(np.uint32), want.view(np.uint32)), (t, r)
        for p in plain:   # the next round's plain aggregates start from zero padding again
            view(p, cap)[:] = 0.0
    for c in encs + srvs + refs:
        c.close()
    for p in land + aggs + plain:
        lib.emu_device_free(p)


def test_emulated_peer_allreduce_sync_one_rank(emu_lib):
    """falcom_peer_allreduce_sync on one emulated rank (its own arrival and
    completion flags release it): the aggregate is unchanged, the flag block
    holds the round number in word 0 (arrival) and word 8 (completion), the
    CTA count is back to 0 and no error is set, for three rounds (a waiter
    compares modulo 2^32, so a round number the flags already passed does
    not wait either); bad arguments are refused."""
    import ctypes
    lib = ctypes.CDLL(emu_lib)
    lib.emu_device_alloc.restype = ctypes.c_void_p
    lib.emu_device_alloc.argtypes = [ctypes.c_size_t]
    lib.emu_device_free.argtypes = [ctypes.c_void_p]
    c_vp = ctypes.c_void_p
    lib.falcom_peer_allreduce_sync.argtypes = [ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), ctypes.c_int,
                                               ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_uint32,
                                               c_vp]
    shard, total = 8192, 8192 - 3
    agg = lib.emu_device_alloc(4 * shard + 256)
    view = np.ctypeslib.as_array((ctypes.c_float * shard).from_address(agg))
    flags = np.ctypeslib.as_array((ctypes.c_uint32 * 64).from_address(agg + 4 * shard))
    x = np.random.default_rng(2).standard_normal(shard).astype(np.float32)
    view[:] = x
    flags[:] = 0
    aggs = (c_vp * 1)(agg)
    fl = (c_vp * 1)(agg + 4 * shard)
    for epoch in (1, 2, 3):
        assert lib.falcom_peer_allreduce_sync(aggs, fl, 1, 0, shard, total, epoch, None) == 0
        assert np.array_equal(view.view(np.uint32), x.view(np.uint32))
        assert flags[0] == epoch and flags[8] == epoch and flags[16] == 0 and flags[17] == 0
    assert lib.falcom_peer_allreduce_sync(aggs, fl, 1, 0, shard, total, 2, None) == 0   # below the flags: passes
    assert flags[17] == 0
    assert lib.falcom_peer_allreduce_sync(aggs, (c_vp * 1)(None), 1, 0, shard, total, 4, None) == -4
    assert lib.falcom_peer_allreduce_sync(aggs, fl, 1, 1, shard, total, 4, None) == -4
    lib.emu_device_free(agg)

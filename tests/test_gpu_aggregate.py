"""GPU tests of the server-side weighted aggregate (falcom_set_aggregate): a
decoder instance that decodes several clients' batches adds each client's
decoded float32 tensors, times the client's weight, into one flat device
buffer.  The aggregate must equal the weighted sum of the decoded outputs the
same calls return (one fma per element and client, so within float32
rounding of the host sum)."""
import ctypes

import numpy as np
import pytest

from compressor_b200.abi import Codec
from tests.helpers import rel_l2, seeded

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SHAPES = [("l1.conv.weight", (64, 32, 3, 3)), ("l1.bn.weight", (64,)), ("l1.bn.bias", (64,)),
          ("l2.conv.weight", (128, 64, 1, 1)), ("fc.weight", (10, 512)), ("fc.bias", (10,)),
          ("l1.bn.num_batches_tracked", (1,))]


def _round_inputs(client, t):
    xs = []
    for i, (name, s) in enumerate(SHAPES):
        if name.endswith("num_batches_tracked"):
            xs.append(np.array([t + 1], np.int64))
        else:
            xs.append(seeded(s, 1000 * client + 10 * t + i))
    return xs


def test_weighted_aggregate_matches_decoded_sum(product_lib):
    names = [n for n, _ in SHAPES]
    sizes = [int(np.prod(s)) for _, s in SHAPES]
    offsets = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sum(sizes))
    nclients = 3
    weights = [0.5, 0.25, 0.25]
    encs = [Codec(product_lib, client=f"c{c}", param_count_threshold=16) for c in range(nclients)]
    server = Codec(product_lib, client="server", param_count_threshold=16)
    off_c = (ctypes.c_size_t * len(names))(*[int(o) for o in offsets])
    for t in range(3):
        agg = torch.zeros(total + 3, dtype=torch.float32, device="cuda")
        want = np.zeros(total, np.float32)
        for c in range(nclients):
            ret, layers, errs = encs[c].compress_batch(names, _round_inputs(c, t))
            assert ret == 0, errs
            assert server.lib.falcom_set_aggregate(server.h, ctypes.c_void_p(agg.data_ptr()), off_c,
                                                   len(names), weights[c]) == 0
            ret, outs = server.decompress_batch(names, layers, client=f"c{c}")
            assert ret == 0
            for i, o in enumerate(outs):
                if o.dtype == np.float32:
                    seg = want[offsets[i]:offsets[i] + sizes[i]]
                    seg[:] = (np.float32(weights[c]) * o.reshape(-1).astype(np.float64) + seg).astype(np.float32)
        torch.cuda.synchronize()
        got = agg.cpu().numpy()
        assert not got[total:].any()                       # nothing written past the last item
        for i, (name, _) in enumerate(SHAPES):
            a, b = got[offsets[i]:offsets[i] + sizes[i]], want[offsets[i]:offsets[i] + sizes[i]]
            if name.endswith("num_batches_tracked"):
                assert not a.any()                         # int64 items are not added
            else:
                assert rel_l2(a, b) <= 1e-6, (name, rel_l2(a, b))
    assert server.lib.falcom_set_aggregate(server.h, None, None, 0, 0.0) == 0
    host = np.zeros(4, np.float32)
    assert server.lib.falcom_set_aggregate(server.h, ctypes.c_void_p(host.ctypes.data), off_c, 1, 1.0) == -4
    for e in encs:
        e.close()
    server.close()


def test_aggregate_with_device_inputs_and_outputs(product_lib):
    """Device-resident inputs, payloads and outputs (the multi-GPU bench's
    path): the aggregate over three rounds equals 2 x the sum of the decoded
    rounds of the same data through the host path."""
    from compressor_b200.abi import PreparedBatch
    names = [n for n, s in SHAPES if not n.endswith("num_batches_tracked")]
    shapes = [s for n, s in SHAPES if not n.endswith("num_batches_tracked")]
    sizes = [int(np.prod(s)) for s in shapes]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    total = int(sum(sizes))
    enc = Codec(product_lib, client="c0", param_count_threshold=16)
    dec = Codec(product_lib, client="c0", param_count_threshold=16)
    henc = Codec(product_lib, client="c0", param_count_threshold=16)
    hdec = Codec(product_lib, client="c0", param_count_threshold=16)
    pb = PreparedBatch(enc.lib, names, shapes)
    agg = torch.zeros(total, dtype=torch.float32, device="cuda")
    off_c = (ctypes.c_size_t * len(names))(*[int(o) for o in offs])
    assert dec.lib.falcom_set_aggregate(dec.h, ctypes.c_void_p(agg.data_ptr()), off_c, len(names), 2.0) == 0
    want = np.zeros(total, np.float32)
    for t in range(3):
        xs = [seeded(s, 77 + 10 * t + i) for i, s in enumerate(shapes)]
        flat = torch.from_numpy(np.concatenate([x.reshape(-1) for x in xs])).cuda()
        torch.cuda.synchronize()
        pb.set_pointers(flat.data_ptr(), [4 * int(o) for o in offs])
        assert pb.compress(enc.h, b"c0") == 0
        assert pb.decompress(dec.h, b"c0") == 0
        torch.cuda.synchronize()
        pb.release()
        ret, layers, _ = henc.compress_batch(names, xs)
        assert ret == 0
        ret, outs = hdec.decompress_batch(names, layers)
        assert ret == 0
        dec_flat = np.concatenate([o.reshape(-1) for o in outs])
        want = (np.float32(2.0) * dec_flat.astype(np.float64) + want).astype(np.float32)
    got = agg.cpu().numpy()
    assert rel_l2(got, want) <= 1e-6, rel_l2(got, want)
    for c in (enc, dec, henc, hdec):
        c.close()


def test_store_mode_equals_clear_then_add(product_lib):
    """falcom_set_aggregate_store: the first client stored (weight * decoded)
    into a buffer full of NaN, the others added, gives the same bits as
    clearing the buffer and adding every client; regions of items that are
    not added (int64) keep their old contents in store mode.  Two rounds."""
    names = [n for n, _ in SHAPES]
    sizes = [int(np.prod(s)) for _, s in SHAPES]
    offsets = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    total = int(sum(sizes))
    weights = [0.5, 0.3, 0.2]
    encs = [Codec(product_lib, client=f"c{c}", param_count_threshold=16) for c in range(3)]
    add_srv = Codec(product_lib, client="server", param_count_threshold=16)
    st_srv = Codec(product_lib, client="server", param_count_threshold=16)
    assert st_srv.lib.falcom_set_aggregate_store(st_srv.h, 2) == -4
    off_c = (ctypes.c_size_t * len(names))(*[int(o) for o in offsets])
    for t in range(2):
        a = torch.zeros(total, dtype=torch.float32, device="cuda")
        b = torch.full((total,), float("nan"), dtype=torch.float32, device="cuda")
        for c in range(3):
            ret, layers, errs = encs[c].compress_batch(names, _round_inputs(c, t))
            assert ret == 0, errs
            for srv, buf in ((add_srv, a), (st_srv, b)):
                assert srv.lib.falcom_set_aggregate(srv.h, ctypes.c_void_p(buf.data_ptr()), off_c, len(names),
                                                    weights[c]) == 0
            assert st_srv.lib.falcom_set_aggregate_store(st_srv.h, 1 if c == 0 else 0) == 0
            assert add_srv.decompress_batch(names, layers, client=f"c{c}")[0] == 0
            assert st_srv.decompress_batch(names, layers, client=f"c{c}")[0] == 0
        torch.cuda.synchronize()
        ga, gb = a.cpu().numpy(), b.cpu().numpy()
        for i, (name, _) in enumerate(SHAPES):
            ra, rb = ga[offsets[i]:offsets[i] + sizes[i]], gb[offsets[i]:offsets[i] + sizes[i]]
            if name.endswith("num_batches_tracked"):
                assert np.isnan(rb).all()                  # not added: left as it was
            else:
                assert np.array_equal(ra.view(np.uint32), rb.view(np.uint32)), name
    assert st_srv.lib.falcom_set_aggregate(st_srv.h, None, None, 0, 0.0) == 0   # also resets the store mode
    for e in encs:
        e.close()


def test_aggregate_only_device_path_exact(product_lib):
    """Aggregate-only decoding (falcom_set_aggregate_only) on device-resident
    inputs and payloads, the federated server's path: no decoded arrays are
    returned, the history still advances, and with two clients of weight 0.5
    (first stored, second added) the aggregate equals 0.5 * (x1 + x2) in
    float32 bit for bit, x1 / x2 being the same clients' decodes from a
    second server that returns arrays.  Three rounds, so rounds 2 and 3
    decode momentum-predicted layers against the aggregate-only server's own
    history."""
    from compressor_b200.abi import PreparedBatch, ndarray_to_numpy
    names = [n for n, s in SHAPES if not n.endswith("num_batches_tracked")]
    shapes = [s for n, s in SHAPES if not n.endswith("num_batches_tracked")]
    sizes = [int(np.prod(s)) for s in shapes]
    # offsets padded to 4 elements (16-byte aligned regions, vector stores)
    offs, o = [], 0
    for n_ in sizes:
        offs.append(o)
        o = (o + n_ + 3) // 4 * 4
    total = o
    encs = [Codec(product_lib, client=f"c{c}", param_count_threshold=16) for c in range(2)]
    srv = Codec(product_lib, client="server", param_count_threshold=16)
    ref = Codec(product_lib, client="server", param_count_threshold=16)
    assert ref.lib.falcom_set_output_location(ref.h, 1) == 0            # decoded arrays in host memory
    pb = PreparedBatch(srv.lib, names, shapes)
    off_c = (ctypes.c_size_t * len(names))(*offs)
    agg = torch.full((total,), float("nan"), dtype=torch.float32, device="cuda")
    for t in range(3):
        decoded = []
        for c in range(2):
            xs = [seeded(s, 900 + 100 * c + 10 * t + i) for i, s in enumerate(shapes)]
            flat = torch.from_numpy(np.concatenate([x.reshape(-1) for x in xs])).cuda()
            torch.cuda.synchronize()
            pb.set_pointers(flat.data_ptr(), [4 * int(v) for v in np.concatenate([[0], np.cumsum(sizes)[:-1]])])
            assert pb.compress(encs[c].h, f"c{c}".encode()) == 0
            assert srv.lib.falcom_set_aggregate(srv.h, ctypes.c_void_p(agg.data_ptr()), off_c, len(names), 0.5) == 0
            assert srv.lib.falcom_set_aggregate_store(srv.h, 1 if c == 0 else 0) == 0
            assert srv.lib.falcom_set_aggregate_only(srv.h, 1) == 0
            assert pb.decompress(srv.h, f"c{c}".encode()) == 0
            assert all(not pb.outs[i] for i in range(len(names)))      # no decoded arrays
            # the same payloads through a server that returns arrays
            rc = ref.lib.momentum_compressor_decompress_batch(ref.h, pb.items, len(names), f"c{c}".encode(),
                                                              pb.outs)
            assert rc == 0
            torch.cuda.synchronize()
            decoded.append([ndarray_to_numpy(pb.outs[i]).reshape(-1).copy() for i in range(len(names))])
            pb.release()
        got = agg.cpu().numpy()
        for i in range(len(names)):
            want = np.float32(0.5) * (decoded[0][i] + decoded[1][i])
            seg = got[offs[i]:offs[i] + sizes[i]]
            assert np.array_equal(seg.view(np.uint32), want.astype(np.float32).view(np.uint32)), (t, names[i])
    assert srv.lib.falcom_set_aggregate_only(srv.h, 2) == -4
    for c in encs + [srv, ref]:
        c.close()

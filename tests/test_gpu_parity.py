"""GPU parity of the B200 codec against the CPU oracle, through the C ABI.

Bar (per the codec's contract):
  * bitmap and dominant-sign bits bit-exact,
  * residual / stats bit-exact in raw mode ("sz3_memcpy"),
  * q8 / int4 codes within +-1 LSB (and in practice identical),
  * decoded update relative L2 <= 1e-6 against the oracle's decoder.
The oracle is the C restatement (oracle/falcom_oracle.c), itself pinned
bit-exact against the reference build in tests/test_oracle_*.py.
"""
import numpy as np
import pytest

from compressor_b200.abi import Codec
from oracle import binding as ob
from tests.helpers import decode_codes, frame_content, rel_l2, seeded

pytestmark = pytest.mark.gpu

SHAPES = [
    ("convA.weight", (64, 64, 3, 3)),     # ks = 9
    ("convB.weight", (128, 64, 1, 1)),    # ks = 1, always predicted
    ("stem.weight", (16, 8, 7, 7)),       # ks = 49
    ("convC.weight", (8, 4, 4, 4)),       # ks = 16 (even)
    ("ragged.weight", (33, 7, 2, 2)),     # ks = 4, K not a multiple of 32
    ("tiny.weight", (2, 2, 2, 2)),        # reference toy shape
    ("five.weight", (5, 3, 5, 5)),        # ks = 25
    ("bn.bias", (64,)),                   # lossless
    ("fc.weight", (10, 512)),             # 2-D lossy, direct_generic
]
THRESHOLD = 4   # momentum path on the toy shapes, as the reference tests do


def make_rounds(n_rounds, seed=0):
    rng = np.random.default_rng(seed)
    out = []
    for t in range(n_rounds):
        r = []
        for i, (_, s) in enumerate(SHAPES):
            x = (rng.standard_normal(s) * 1e-3).astype(np.float32)
            if i == 5 and t == 2:
                x[:] = 0.0                     # all zeros: ties, dominant +1
            if i == 6:
                x.reshape(-1)[:: 3 + t] = 0.0  # zeros counted with the majority
            r.append(x)
        out.append(r)
    return out


class OracleClient:
    """Encoder + decoder state of the CPU oracle for one client."""

    def __init__(self, qmax):
        self.qmax = qmax
        self.prev = {}
        self.mem = {}
        self.dprev = {}
        self.dmem = {}

    def encode(self, name, x, step):
        shape = x.shape
        if step == 1 or name not in self.prev or not (len(shape) == 4 and x.size > THRESHOLD
                                                      and "weight" in name):
            self.prev[name] = x.copy()
            return None
        mem = self.mem.setdefault(name, np.zeros(x.size, np.float32))
        o = ob.encode_momentum(x, self.prev[name], mem, step=step)
        self.prev[name] = x.copy()
        return o


@pytest.mark.parametrize("codec", ["raw", "q8", "int4"])
def test_encoder_decoder_match_oracle(product_lib, codec):
    enc = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    dec = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    assert enc.lib.falcom_set_residual_codec(enc.h, codec.encode()) == 0
    qmax = {"raw": 0, "q8": 127, "int4": 7}[codec]
    orc = OracleClient(qmax)
    names = [n for n, _ in SHAPES]
    data = make_rounds(4)
    dmem, dprev = {}, {}
    for t, xs in enumerate(data):
        ret, layers, errs = enc.compress_batch(names, xs)
        assert ret == 0, (ret, errs, enc.lib.falcom_last_error(enc.h))
        for (name, shape), x, L in zip(SHAPES, xs, layers):
            step = t + 1
            assert L.step == step
            o = orc.encode(name, x, step)
            if o is None:
                assert L.type == ("direct" if step == 1 else "direct_generic"), (name, L.type)
                if "weight" in name and x.size > THRESHOLD:
                    if codec == "raw":
                        assert L.codec == "sz3_memcpy"
                        assert L.data == x.tobytes()
                    else:
                        scale, codes = decode_codes(L, x.size)
                        es, ec = ob.quantize(x, qmax)
                        assert scale == es
                        assert np.array_equal(codes, ec)
                else:
                    assert L.codec == "zstd"
                    assert frame_content(L.data) == x.tobytes()
                continue
            assert L.type == "momentum_predicted", (name, L.type)
            st = o["stats"]
            assert frame_content(L.bitmap) == o["bitmap"].tobytes(), name
            assert frame_content(L.dominant_signs) == o["signs"].tobytes(), name
            assert L.num_predicted_kernels == st["predicted"]
            assert (L.current_mean, L.current_std, L.prev_mean, L.prev_std) == (
                st["cur_mean"], st["cur_std"], st["prev_mean"], st["prev_std"]), name
            assert (L.global_min, L.global_max) == (st["gmin"], st["gmax"])
            assert L.prediction_ratio == st["prediction_ratio"]
            assert L.sign_mismatch_ratio == st["sign_mismatch_ratio"]
            if codec == "raw":
                got = np.frombuffer(L.data, np.float32)
                assert np.array_equal(got.view(np.uint32), o["residual"].view(np.uint32)), name
            else:
                scale, codes = decode_codes(L, x.size)
                es, ec = ob.quantize(o["residual"], qmax)
                assert scale == es, name
                assert np.max(np.abs(codes.astype(int) - ec.astype(int))) <= 1, name
                assert np.array_equal(codes, ec), name

        # decoder: ours against the oracle decoder fed with the same payload
        ret, outs = dec.decompress_batch(names, layers)
        assert ret == 0
        for (name, shape), L, y in zip(SHAPES, layers, outs):
            assert y is not None and y.shape == shape
            if L.type == "momentum_predicted":
                if L.codec == "sz3_memcpy":
                    res = np.frombuffer(L.data, np.float32)
                else:
                    scale, codes = decode_codes(L, int(np.prod(shape)))
                    res = ob.dequantize(codes, scale)
                mem = dmem.setdefault(name, np.zeros(int(np.prod(shape)), np.float32))
                exp, appended = ob.decode_momentum(
                    res, frame_content(L.bitmap), frame_content(L.dominant_signs) or None,
                    dprev.get(name), mem, shape, L.current_mean, L.current_std, L.prev_mean,
                    L.prev_std)
                assert rel_l2(exp, y) <= 1e-6, name
                assert np.array_equal(exp.view(np.uint32), y.view(np.uint32)), name
                if appended:
                    dprev[name] = exp.copy()
            else:
                if L.codec in ("q8", "int4"):
                    scale, codes = decode_codes(L, int(np.prod(shape)))
                    exp = ob.dequantize(codes, scale).reshape(shape)
                else:
                    exp = data[t][names.index(name)]
                assert np.array_equal(exp.view(np.uint32), y.view(np.uint32)), name
                dprev[name] = exp.copy()
    enc.close()
    dec.close()


def test_against_reference_build_raw(product_lib):
    """Same seeded batches through the reference library (built from the
    reference's own sources) and through this codec in raw mode."""
    if not ob.have_ref():
        pytest.skip("reference build oracle/_ref not present")
    ours = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    ref = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    ours_d = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    ref_d = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    ours.lib.falcom_set_residual_codec(ours.h, b"raw")
    names = [n for n, _ in SHAPES]
    for t, xs in enumerate(make_rounds(4, seed=5)):
        r1, A, _ = ours.compress_batch(names, xs)
        r2, B, _ = ref.compress_batch(names, xs)
        assert r1 == 0 and r2 == 0
        for a, b in zip(A, B):
            assert (a.type, a.step, a.shape, a.original_dtype, a.stored_dtype) == (
                b.type, b.step, b.shape, b.original_dtype, b.stored_dtype)
            if a.codec == "sz3_memcpy":
                assert b.codec == "sz3_memcpy" and a.data == b.data
            else:
                assert frame_content(a.data) == frame_content(b.data)
            assert frame_content(a.bitmap) == frame_content(b.bitmap)
            assert frame_content(a.dominant_signs) == frame_content(b.dominant_signs)
            assert (a.current_mean, a.current_std, a.prev_mean, a.prev_std, a.global_min,
                    a.global_max, a.num_predicted_kernels, a.prediction_ratio,
                    a.sign_mismatch_ratio) == (
                b.current_mean, b.current_std, b.prev_mean, b.prev_std, b.global_min,
                b.global_max, b.num_predicted_kernels, b.prediction_ratio, b.sign_mismatch_ratio)
        # cross decode: each decoder reads the other's payloads
        ra, YA = ours_d.decompress_batch(names, B)
        rb, YB = ref_d.decompress_batch(names, A)
        assert ra == 0 and rb == 0
        for ya, yb in zip(YA, YB):
            assert np.array_equal(ya.view(np.uint32), yb.view(np.uint32))


def test_libzstd_frames_byte_identical_to_reference(product_lib):
    if not ob.have_ref():
        pytest.skip("reference build oracle/_ref not present")
    ours = Codec(product_lib, client="client_0", param_count_threshold=THRESHOLD)
    ref = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    ours.lib.falcom_set_residual_codec(ours.h, b"raw")
    assert ours.lib.falcom_set_frame_mode(ours.h, b"libzstd") == 0
    names = [n for n, _ in SHAPES]
    for xs in make_rounds(3, seed=9):
        _, A, _ = ours.compress_batch(names, xs)
        _, B, _ = ref.compress_batch(names, xs)
        for a, b in zip(A, B):
            assert a.bitmap == b.bitmap
            assert a.dominant_signs == b.dominant_signs
            assert a.data == b.data
            size_a = len(a.data) + len(a.bitmap) + len(a.dominant_signs)
            size_b = len(b.data) + len(b.bitmap) + len(b.dominant_signs)
            assert size_a == size_b   # compression ratio identical


def test_gpu_frames_are_valid_zstd(product_lib):
    c = Codec(product_lib, client="c", param_count_threshold=THRESHOLD)
    names = ["big.weight", "ones.weight"]
    xs0 = [seeded((256, 256, 3, 3), 1), np.ones((1024, 300, 1, 1), np.float32)]
    xs1 = [seeded((256, 256, 3, 3), 2), np.ones((1024, 300, 1, 1), np.float32)]
    c.compress_batch(names, xs0)
    _, L, _ = c.compress_batch(names, xs1)
    for layer in L:
        bm = ob.zstd_decompress(layer.bitmap)
        assert len(bm) == (layer.shape[0] * layer.shape[1] + 7) // 8
    # all-ones bitmap of 1x1 kernels: RLE blocks keep the frame tiny
    assert len(L[1].bitmap) < 64

"""Encoder/decoder parity cases shared by the GPU tests and the CPU kernel
emulation tests: seeded batches of conv/linear/bias shapes covering every
kernel size class, ragged kernel counts, all-zero and zero-heavy tensors, run
through the library's C ABI and checked against the CPU oracle.

Bar (per the codec's contract):
  * bitmap and dominant-sign bits bit-exact,
  * residual / stats bit-exact in raw mode ("sz3_memcpy"),
  * q8 / int4 codes within +-1 LSB (and in practice identical),
  * decoded update relative L2 <= 1e-6 against the oracle's decoder.
"""
import numpy as np

from compressor_b200.abi import Codec
from oracle import binding as ob
from tests.helpers import decode_codes, frame_content, rel_l2

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
    ("head.weight", (9, 1001)),           # 2-D lossy, ragged: an 8192-element encoder tile plus 817
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


def check_encoder_decoder(lib_path, codec, n_rounds=4, seed=0):
    """Encodes n_rounds seeded batches of SHAPES with the library at lib_path
    and decodes them again, checking every payload and every decoded tensor
    against the oracle."""
    enc = Codec(lib_path, client="client_0", param_count_threshold=THRESHOLD)
    dec = Codec(lib_path, client="client_0", param_count_threshold=THRESHOLD)
    assert enc.lib.falcom_set_residual_codec(enc.h, codec.encode()) == 0
    qmax = {"raw": 0, "q8": 127, "int4": 7, "q8_raw": 127, "int4_raw": 7}[codec]
    # raw, q8_raw and int4_raw store fp32 payloads under the tag "sz3_memcpy":
    # the values themselves, or the quantised values dequantised
    float_payload = codec in ("raw", "q8_raw", "int4_raw")

    def payload_floats(v):
        if codec == "raw":
            return np.ascontiguousarray(v, np.float32).reshape(-1)
        es, ec = ob.quantize(v, qmax)
        return ob.dequantize(ec, es)

    orc = OracleClient(qmax)
    names = [n for n, _ in SHAPES]
    data = make_rounds(n_rounds, seed)
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
                    if float_payload:
                        assert L.codec == "sz3_memcpy"
                        got = np.frombuffer(L.data, np.float32)
                        assert np.array_equal(got.view(np.uint32), payload_floats(x).view(np.uint32)), name
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
            if float_payload:
                assert L.codec == "sz3_memcpy", name
                got = np.frombuffer(L.data, np.float32)
                assert np.array_equal(got.view(np.uint32), payload_floats(o["residual"]).view(np.uint32)), name
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
                elif L.codec == "sz3_memcpy":
                    exp = np.frombuffer(L.data, np.float32).reshape(shape)
                else:
                    exp = data[t][names.index(name)]
                assert np.array_equal(exp.view(np.uint32), y.view(np.uint32)), name
                dprev[name] = exp.copy()
    enc.close()
    dec.close()

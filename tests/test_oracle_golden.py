"""Pins the CPU restatement oracle against the reference's recorded outputs
(tests/golden/reference_vectors.npz, written by tests/golden/make_golden.py
from the reference library built from its own sources)."""
import os

import numpy as np
import pytest

from oracle import binding as ob

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_vectors.npz")
THRESHOLD = 4


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def stats_array(st):
    return np.array([st["cur_mean"], st["cur_std"], st["prev_mean"], st["prev_std"], st["gmin"],
                     st["gmax"], st["prediction_ratio"], st["sign_mismatch_ratio"]], np.float32)


def test_encoder_and_decoder_match_reference_vectors(gold, oracle_lib):
    names = list(gold["names"])
    R = int(gold["rounds"])
    prev, mem, dprev, dmem = {}, {}, {}, {}
    checked = 0
    for t in range(R):
        for i, name in enumerate(names):
            k = f"r{t}_l{i}_"
            x = gold[k + "input"]
            typ = str(gold[k + "type"])
            assert int(gold[k + "step"]) == t + 1
            if typ != "momentum_predicted":
                # direct payloads are the raw input bytes (zstd content for lossless)
                assert gold[k + "data"].tobytes() == x.tobytes()
                assert np.array_equal(gold[k + "decoded"].view(np.uint32), x.view(np.uint32))
                prev[name] = x.copy()
                dprev[name] = x.copy()
                continue
            m = mem.setdefault(name, np.zeros(x.size, np.float32))
            o = ob.encode_momentum(x, prev[name], m, step=t + 1)
            prev[name] = x.copy()
            assert gold[k + "bitmap"].tobytes() == o["bitmap"].tobytes(), k
            assert gold[k + "signs"].tobytes() == o["signs"].tobytes(), k
            assert np.array_equal(gold[k + "stats"], stats_array(o["stats"])), k
            assert int(gold[k + "num_predicted"]) == o["stats"]["predicted"]
            res = np.frombuffer(gold[k + "data"].tobytes(), np.float32)
            assert np.array_equal(res.view(np.uint32), o["residual"].view(np.uint32)), k
            st = gold[k + "stats"]
            dm = dmem.setdefault(name, np.zeros(x.size, np.float32))
            rec, appended = ob.decode_momentum(res, gold[k + "bitmap"].tobytes(),
                                               gold[k + "signs"].tobytes() or None, dprev[name], dm,
                                               x.shape, st[0], st[1], st[2], st[3])
            assert np.array_equal(rec.view(np.uint32), gold[k + "decoded"].view(np.uint32)), k
            if appended:
                dprev[name] = rec.copy()
            checked += 1
    assert checked >= 15


def test_state_oracle_chain_vectors(gold, oracle_lib):
    xs = [gold[f"chain{j}_input"] for j in range(3)]
    assert str(gold["chain0_type"]) == "direct"
    assert [int(gold[f"chain{j}_step"]) for j in range(3)] == [1, 2, 3]
    mem = np.zeros(16, np.float32)
    for j in (1, 2):
        o = ob.encode_momentum(xs[j], xs[j - 1], mem, step=j + 1)
        assert str(gold[f"chain{j}_type"]) == "momentum_predicted"
        assert gold[f"chain{j}_bitmap"].tobytes() == o["bitmap"].tobytes()
        assert gold[f"chain{j}_signs"].tobytes() == o["signs"].tobytes()
        res = np.frombuffer(gold[f"chain{j}_data"].tobytes(), np.float32)
        assert np.array_equal(res.view(np.uint32), o["residual"].view(np.uint32))


def test_quantiser_known_answers(oracle_lib):
    # q8: scale = max|x|/127, round half to even, clamp
    x = np.array([0.0, 1.0, -1.0, 0.5, -0.25, 127 / 254.0], np.float32)
    scale, codes = ob.quantize(x, 127)
    assert scale == np.float32(1.0) / np.float32(127.0)
    assert list(codes[:5]) == [0, 127, -127, 64, -32]   # 63.5 -> 64, -31.75 -> -32
    assert codes[5] == 64                               # 63.5 rounds to even
    # all zeros: scale 1, codes 0
    s0, c0 = ob.quantize(np.zeros(7, np.float32), 127)
    assert s0 == 1.0 and not c0.any()
    # int4: qmax 7, (q+8) nibbles, element 2i low
    s4, c4 = ob.quantize(np.array([-7, 7, 3.5, 0, 1], np.float32), 7)
    assert s4 == 1.0 and list(c4) == [-7, 7, 4, 0, 1]
    packed = ob.pack_int4(c4)
    assert list(packed) == [(1) | (15 << 4), (12) | (8 << 4), 9]
    assert list(ob.unpack_int4(packed, 5)) == list(c4)


def test_consistency_threshold_boundaries(oracle_lib):
    """ks = 4 with 3 of 4 positive is exactly 0.5 (predicted); ks = 9 needs 7."""
    flags = np.zeros(4, np.uint8)
    dom = np.zeros(4, np.int8)
    cur = np.array([1, 1, 1, -1,   1, 1, -1, -1,   0, 0, 0, 0,   -1, -1, -1, 0], np.float32)
    P = ob.lib().fo_sign_consistency(cur, 4, 4, 0.5, flags, dom)
    assert list(flags) == [1, 0, 1, 1] and P == 3
    assert list(dom) == [1, 1, 1, -1]       # ties -> +1; zeros join the majority
    cur9 = np.array([1] * 6 + [-1] * 3 + [1] * 7 + [-1] * 2, np.float32)
    f9 = np.zeros(2, np.uint8)
    d9 = np.zeros(2, np.int8)
    ob.lib().fo_sign_consistency(cur9, 2, 9, 0.5, f9, d9)
    assert list(f9) == [0, 1]

"""Generates tests/golden/reference_vectors.npz from the reference codec.

Runs the reference library built from the reference's own sources
(oracle/_ref/libmomentum_compressor_ref.so; SZ3 absent, so residuals come out
as raw "sz3_memcpy" floats) on small seeded inputs through its C ABI: a
4-round closed loop over layers with kernel sizes 1, 4, 9, 16, 25, 49 plus
lossless and 2-D tensors, with a separate decoder instance, and the step chain
of the reference's own state-oracle test inputs.  Every payload and decoded
output is stored, so the CPU oracle and the GPU codec can be checked against
the reference without the reference being present.

Usage (needs oracle/_ref, i.e. the reference checkout when building):
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from compressor_b200.abi import Codec  # noqa: E402
from oracle import binding as ob  # noqa: E402

SHAPES = [
    ("l0.conv.weight", (16, 16, 3, 3)),
    ("l1.conv.weight", (32, 16, 1, 1)),
    ("l2.conv.weight", (4, 4, 7, 7)),
    ("l3.conv.weight", (8, 4, 4, 4)),
    ("l4.conv.weight", (33, 7, 2, 2)),
    ("l5.conv.weight", (2, 2, 2, 2)),
    ("l6.conv.weight", (5, 3, 5, 5)),
    ("l7.bn.bias", (16,)),
    ("l8.fc.weight", (10, 64)),
]
ROUNDS = 4
THRESHOLD = 4


def inputs():
    rng = np.random.Generator(np.random.PCG64(20261201))
    out = []
    for t in range(ROUNDS):
        r = []
        for i, (_, s) in enumerate(SHAPES):
            x = (rng.standard_normal(s) * 1e-3).astype(np.float32)
            if i == 6:
                x.reshape(-1)[:: 3 + t] = 0.0
            if i == 5 and t == 2:
                x[:] = 0.0
            r.append(x)
        out.append(r)
    return out


def state_oracle_inputs():
    """The sin/cos input formula of the reference's state-oracle test
    (float32, seeds 1..3, 2x2x2x2)."""
    res = []
    for seed in (1, 2, 3):
        i = np.arange(16, dtype=np.float32)
        x = (np.sin((i + 1) * np.float32(0.13) + np.float32(seed) * np.float32(0.17)) +
             np.cos((i + 3) * np.float32(0.05) - np.float32(seed) * np.float32(0.11)))
        res.append(x.astype(np.float32).reshape(2, 2, 2, 2))
    return res


def main():
    if not ob.have_ref():
        sys.exit("oracle/_ref/libmomentum_compressor_ref.so is missing (make -C oracle ref)")
    enc = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    dec = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    names = [n for n, _ in SHAPES]
    rec = {"names": np.array(names), "rounds": np.int64(ROUNDS)}
    for t, xs in enumerate(inputs()):
        ret, layers, errs = enc.compress_batch(names, xs)
        assert ret == 0, (ret, errs)
        ret2, outs = dec.decompress_batch(names, layers)
        assert ret2 == 0
        for i, (x, L, y) in enumerate(zip(xs, layers, outs)):
            k = f"r{t}_l{i}_"
            rec[k + "input"] = x
            rec[k + "type"] = np.array(L.type)
            rec[k + "codec"] = np.array(L.codec)
            rec[k + "step"] = np.int64(L.step)
            data = ob.zstd_decompress(L.data) if L.codec == "zstd" else L.data
            rec[k + "data"] = np.frombuffer(data, np.uint8)
            rec[k + "bitmap"] = np.frombuffer(ob.zstd_decompress(L.bitmap) if L.bitmap else b"", np.uint8)
            rec[k + "signs"] = np.frombuffer(ob.zstd_decompress(L.dominant_signs) if L.dominant_signs else b"", np.uint8)
            rec[k + "stats"] = np.array([L.current_mean, L.current_std, L.prev_mean, L.prev_std,
                                         L.global_min, L.global_max, L.prediction_ratio,
                                         L.sign_mismatch_ratio], np.float32)
            rec[k + "num_predicted"] = np.int64(L.num_predicted_kernels)
            rec[k + "decoded"] = y
    # step chain of the reference state-oracle inputs, one instance, serial batch
    os.environ["FALCOM_BATCH_SERIAL"] = "1"
    chain = Codec(ob.REF_SO, client="client_0", param_count_threshold=THRESHOLD)
    xs = state_oracle_inputs()
    ret, layers, _ = chain.compress_batch(["convA.weight"] * 3, xs)
    del os.environ["FALCOM_BATCH_SERIAL"]
    assert ret == 0
    for j, (x, L) in enumerate(zip(xs, layers)):
        k = f"chain{j}_"
        rec[k + "input"] = x
        rec[k + "type"] = np.array(L.type)
        rec[k + "step"] = np.int64(L.step)
        rec[k + "data"] = np.frombuffer(L.data, np.uint8)
        rec[k + "bitmap"] = np.frombuffer(ob.zstd_decompress(L.bitmap) if L.bitmap else b"", np.uint8)
        rec[k + "signs"] = np.frombuffer(ob.zstd_decompress(L.dominant_signs) if L.dominant_signs else b"", np.uint8)
        rec[k + "stats"] = np.array([L.current_mean, L.current_std, L.prev_mean, L.prev_std,
                                     L.global_min, L.global_max, L.prediction_ratio,
                                     L.sign_mismatch_ratio], np.float32)
    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **rec)
    print("wrote", len(rec), "arrays")


if __name__ == "__main__":
    main()

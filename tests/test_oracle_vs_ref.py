"""Pins the CPU restatement oracle against the reference build itself
(oracle/_ref, compiled from the reference's own sources here) on random
inputs, and runs the reference's own C contract tests against that build.
Skipped where the reference build is absent."""
import os
import subprocess

import numpy as np
import pytest

from compressor_b200.abi import Codec
from oracle import binding as ob

pytestmark = pytest.mark.skipif(not ob.have_ref(), reason="reference build oracle/_ref not present")

SHAPES = [(64, 64, 3, 3), (128, 64, 1, 1), (16, 8, 7, 7), (8, 4, 4, 4), (33, 7, 2, 2), (2, 2, 2, 2),
          (5, 3, 5, 5), (3, 3, 3, 1)]


@pytest.mark.parametrize("seed", [0, 1])
def test_restatement_bit_exact_vs_reference(seed, oracle_lib):
    rng = np.random.default_rng(seed)
    names = [f"layer{i}.conv.weight" for i in range(len(SHAPES))]
    enc = Codec(ob.REF_SO, client="client_0", param_count_threshold=4)
    dec = Codec(ob.REF_SO, client="client_0", param_count_threshold=4)
    mems = [np.zeros(int(np.prod(s)), np.float32) for s in SHAPES]
    dmems = [np.zeros(int(np.prod(s)), np.float32) for s in SHAPES]
    dprev = [None] * len(SHAPES)
    prev = None
    for t in range(4):
        data = [(rng.standard_normal(s) * 10 ** rng.uniform(-5, 0)).astype(np.float32) for s in SHAPES]
        if t == 2:
            data[5][:] = 0
        ret, layers, _ = enc.compress_batch(names, data)
        ret2, outs = dec.decompress_batch(names, layers)
        assert ret == 0 and ret2 == 0
        for i, (s, L) in enumerate(zip(SHAPES, layers)):
            if t == 0:
                dprev[i] = data[i]
                continue
            o = ob.encode_momentum(data[i], prev[i], mems[i], step=t + 1)
            st = o["stats"]
            assert ob.zstd_decompress(L.bitmap) == o["bitmap"].tobytes()
            assert (ob.zstd_decompress(L.dominant_signs) if L.dominant_signs else b"") == o["signs"].tobytes()
            res = np.frombuffer(L.data, np.float32)
            assert np.array_equal(res.view(np.uint32), o["residual"].view(np.uint32))
            assert (L.current_mean, L.current_std, L.prev_mean, L.prev_std) == (
                st["cur_mean"], st["cur_std"], st["prev_mean"], st["prev_std"])
            rec, app = ob.decode_momentum(res, ob.zstd_decompress(L.bitmap),
                                          ob.zstd_decompress(L.dominant_signs) if L.dominant_signs else None,
                                          dprev[i], dmems[i], s, L.current_mean, L.current_std,
                                          L.prev_mean, L.prev_std)
            assert np.array_equal(rec.view(np.uint32), outs[i].view(np.uint32))
            if app:
                dprev[i] = rec
        prev = data


@pytest.mark.parametrize("prog", ["test_reference_state_oracle", "test_batch_state_equivalence",
                                  "test_runtime_contracts"])
def test_reference_c_contract_programs_pass_on_reference_build(prog):
    exe = os.path.join(os.path.dirname(ob.REF_SO), prog)
    if not os.path.exists(exe):
        pytest.skip("reference test program not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "ok - " in r.stdout

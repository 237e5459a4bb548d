"""Replay rounds on the GPU and the state checkpoint.

* A round loaded into device memory holds the same bytes as the file (written
  back from the device items), and compress_batch on the device items gives
  the same payloads as on the host arrays.
* falcom_state_save / falcom_state_load: an encoder and a decoder restored
  from a checkpoint into fresh instances continue with exactly the payloads /
  outputs the saved instances produce; a file that is not a checkpoint is
  refused and leaves the state as it was."""
import ctypes
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from compressor_b200 import replay
from compressor_b200 import workloads as W
from compressor_b200.abi import Codec, Layer

pytestmark = pytest.mark.gpu


def _rounds(model, n, seed=5):
    lay = W.Layout.of(model)
    return lay, [lay.views(f) for f in W.rounds(model, n, seed=seed)]


def _same(a, b):
    assert (a.type, a.codec, a.step, a.shape, a.data, a.bitmap, a.dominant_signs) == \
        (b.type, b.codec, b.step, b.shape, b.data, b.bitmap, b.dominant_signs)
    assert (a.current_mean, a.current_std, a.prev_mean, a.prev_std, a.num_predicted_kernels) == \
        (b.current_mean, b.current_std, b.prev_mean, b.prev_std, b.num_predicted_kernels)


def test_device_replay_matches_file_and_host_path(tmp_path, product_lib):
    lay, rounds = _rounds("resnet18", 2)
    paths = []
    for t, xs in enumerate(rounds):
        p = str(tmp_path / f"round{t}.bin")
        assert replay.write_round(p, t, "Client1", dict(zip(lay.names, xs)), product_lib) == 0
        paths.append(p)
    host = Codec(product_lib, client="Client1")
    dev = Codec(product_lib, client="Client1")
    assert dev.lib.falcom_set_payload_location(dev.h, 1) == 0    # host payloads, to compare
    for t, p in enumerate(paths):
        with replay.ReplayRound(p, "device", 0, product_lib) as r:
            assert r.n == len(lay.names) and r.round == t and r.client == "Client1"
            assert all(dev.lib.falcom_is_device_pointer(ctypes.c_void_p(q)) for q in r.ptrs)
            # the device copy holds the file's bytes
            back = str(tmp_path / f"back{t}.bin")
            assert r.lib.falcom_replay_write(back.encode(), t, b"Client1", r.items, r.n) == 0
            assert open(back, "rb").read() == open(p, "rb").read()
            ret = dev.lib.momentum_compressor_compress_batch(dev.h, r.items, r.n, b"Client1")
            assert ret == 0
            got = [Layer.from_c(r.items[i].compressed.contents) for i in range(r.n)]
            for i in range(r.n):
                dev.lib.compressed_layer_data_free(r.items[i].compressed)
                r.items[i].compressed = None
        ret, want, _ = host.compress_batch(lay.names, rounds[t])
        assert ret == 0
        for name, a, b in zip(lay.names, got, want):
            _same(a, b)
    host.close()
    dev.close()


def test_checkpoint_resumes_encoder_and_decoder(tmp_path, product_lib):
    lay, rounds = _rounds("resnet18", 4, seed=11)
    enc_a = Codec(product_lib, client="Client1")
    dec_a = Codec(product_lib, client="Client1")
    payloads = []
    for t in range(2):
        ret, L, _ = enc_a.compress_batch(lay.names, rounds[t])
        assert ret == 0
        payloads.append(L)
        ret, _ = dec_a.decompress_batch(lay.names, L)
        assert ret == 0
    ck_enc, ck_dec = str(tmp_path / "enc.fcst"), str(tmp_path / "dec.fcst")
    assert enc_a.save_state(ck_enc) == 0
    assert dec_a.save_state(ck_dec) == 0
    # the saved instances continue ...
    want = []
    for t in (2, 3):
        ret, L, _ = enc_a.compress_batch(lay.names, rounds[t])
        assert ret == 0
        want.append(L)
    assert any(l.type == "momentum_predicted" for l in want[0])
    out_a = []
    for L in want:
        ret, Y = dec_a.decompress_batch(lay.names, L)
        assert ret == 0
        out_a.append(Y)
    # ... and so do fresh instances restored from the checkpoints
    enc_b = Codec(product_lib, client="Client1")
    dec_b = Codec(product_lib, client="Client1")
    assert enc_b.load_state(ck_enc) == 0
    assert dec_b.load_state(ck_dec) == 0
    for t, L_want in zip((2, 3), want):
        ret, L, _ = enc_b.compress_batch(lay.names, rounds[t])
        assert ret == 0
        for a, b in zip(L, L_want):
            _same(a, b)
    for L, Y_want in zip(want, out_a):
        ret, Y = dec_b.decompress_batch(lay.names, L)
        assert ret == 0
        for y, z in zip(Y, Y_want):
            assert np.array_equal(y.view(np.uint8), z.view(np.uint8))
    for c in (enc_a, dec_a, enc_b, dec_b):
        c.close()


def test_checkpoint_refuses_other_files(tmp_path, product_lib):
    lay, rounds = _rounds("resnet18", 2, seed=3)
    enc = Codec(product_lib, client="Client1")
    ret, L0, _ = enc.compress_batch(lay.names, rounds[0])
    assert ret == 0
    bad = tmp_path / "bad.fcst"
    bad.write_bytes(b"FCSTATE1" + b"\x07" * 40)
    assert enc.load_state(str(bad)) != 0
    assert enc.load_state(str(tmp_path / "missing.fcst")) != 0
    good = str(tmp_path / "good.fcst")
    assert enc.save_state(good) == 0
    raw = open(good, "rb").read()
    (tmp_path / "cut.fcst").write_bytes(raw[:len(raw) // 2])
    assert enc.load_state(str(tmp_path / "cut.fcst")) != 0
    assert enc.save_state(str(tmp_path / "no_dir" / "x.fcst")) != 0
    # the refused loads left the state alone: round 1 continues from round 0
    ret, L1, _ = enc.compress_batch(lay.names, rounds[1])
    assert ret == 0
    ref = Codec(product_lib, client="Client1")
    assert ref.compress_batch(lay.names, rounds[0])[0] == 0
    ret, R1, _ = ref.compress_batch(lay.names, rounds[1])
    for a, b in zip(L1, R1):
        _same(a, b)
    enc.close()
    ref.close()


def test_bench_replay_mode(tmp_path, product_lib):
    lay, rounds = _rounds("resnet18", 3, seed=9)
    for t, xs in enumerate(rounds):
        t_all = dict(zip(lay.names, xs))
        t_all["bn1.num_batches_tracked"] = np.array(t + 1, dtype=np.int64)   # scalars are left out
        assert replay.write_round(str(tmp_path / f"r{t}.bin"), t, "Client3", t_all, product_lib) == 0
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--replay", str(tmp_path / "r*.bin"),
                          "--steps", "3", "--warmup", "3"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["unit"] == "GB/s" and line["value"] > 0 and line["steps"] == 3
    assert line["config"]["client"] == "Client3"

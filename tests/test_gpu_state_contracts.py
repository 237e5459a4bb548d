"""Reference contract tests (test_reference_state_oracle.c,
test_batch_state_equivalence.c, test_runtime_contracts.c) restated over the
C ABI of the B200 codec, plus the reference programs themselves linked
against this library when they were built."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from compressor_b200.abi import Codec, Layer
from oracle import binding as ob

pytestmark = pytest.mark.gpu
THR = 4


def sincos(shape, seed):
    i = np.arange(int(np.prod(shape)), dtype=np.float32)
    x = (np.sin((i + 1) * np.float32(0.13) + np.float32(seed) * np.float32(0.17)) +
         np.cos((i + 3) * np.float32(0.05) - np.float32(seed) * np.float32(0.11)))
    return x.astype(np.float32).reshape(shape)


def serial(monkeypatch):
    monkeypatch.setenv("FALCOM_BATCH_SERIAL", "1")
    monkeypatch.delenv("FALCOM_BATCH_PARALLEL", raising=False)


def grouped(monkeypatch):
    monkeypatch.delenv("FALCOM_BATCH_SERIAL", raising=False)
    monkeypatch.setenv("FALCOM_BATCH_PARALLEL", "1")


@pytest.mark.parametrize("mode", [serial, grouped])
def test_repeated_layer_step_chain(product_lib, monkeypatch, mode):
    mode(monkeypatch)
    c = Codec(product_lib, client="client_0", param_count_threshold=THR)
    xs = [sincos((2, 2, 2, 2), s) for s in (1, 2, 3)]
    ret, layers, _ = c.compress_batch(["convA.weight"] * 3, xs)
    assert ret == 0
    assert [L.step for L in layers] == [1, 2, 3]
    assert [L.type for L in layers] == ["direct", "momentum_predicted", "momentum_predicted"]
    for L in layers:
        y = c.decompress_layer(L, "convA.weight")
        assert y is not None and np.all(np.isfinite(y))


def test_grouped_chain_matches_serial_chain(product_lib, monkeypatch):
    """Repeated layers in one grouped batch chain their memory exactly like
    the serial path (memory waves)."""
    xs = [sincos((4, 3, 3, 3), s) for s in (1, 2, 3, 4)]
    out = {}
    for name, mode in (("serial", serial), ("grouped", grouped)):
        mode(monkeypatch)
        c = Codec(product_lib, client="client_0", param_count_threshold=THR)
        c.lib.falcom_set_residual_codec(c.h, b"raw")
        ret, layers, _ = c.compress_batch(["convA.weight"] * 4, xs)
        assert ret == 0
        out[name] = layers
    for a, b in zip(out["serial"], out["grouped"]):
        assert a.type == b.type and a.step == b.step
        assert a.data == b.data and a.bitmap == b.bitmap and a.dominant_signs == b.dominant_signs


def test_interleaved_layers_independent_steps(product_lib, monkeypatch):
    serial(monkeypatch)
    c = Codec(product_lib, client="client_0", param_count_threshold=THR)
    names = ["convA.weight", "fcB.bias", "convA.weight", "bnC.bias", "fcB.bias", "convA.weight"]
    xs = [sincos((2, 2, 2, 2) if "conv" in n else (8,), i + 10) for i, n in enumerate(names)]
    ret, layers, _ = c.compress_batch(names, xs)
    assert ret == 0
    assert [L.step for L in layers] == [1, 1, 2, 1, 2, 3]


@pytest.mark.parametrize("mode", [serial, grouped])
def test_same_shape_layers_are_independent(product_lib, monkeypatch, mode):
    mode(monkeypatch)
    shared = Codec(product_lib, client="client_0", param_count_threshold=THR)
    a_only = Codec(product_lib, client="client_0", param_count_threshold=THR)
    b_only = Codec(product_lib, client="client_0", param_count_threshold=THR)
    for r in range(3):
        xa, xb = sincos((2, 2, 2, 2), 100 + r), sincos((2, 2, 2, 2), 200 + r)
        _, S, _ = shared.compress_batch(["convA.weight", "convB.weight"], [xa, xb])
        _, A, _ = a_only.compress_batch(["convA.weight"], [xa])
        _, B, _ = b_only.compress_batch(["convB.weight"], [xb])
        assert (S[0].data, S[0].bitmap, S[0].dominant_signs) == (A[0].data, A[0].bitmap, A[0].dominant_signs)
        assert (S[1].data, S[1].bitmap, S[1].dominant_signs) == (B[0].data, B[0].bitmap, B[0].dominant_signs)


def test_shape_change_never_reuses_history(product_lib, monkeypatch):
    serial(monkeypatch)
    c = Codec(product_lib, client="client_0", param_count_threshold=THR)
    xs = [sincos((2, 2, 2, 2), 301), sincos((3, 2, 2, 2), 302), sincos((2, 2, 2, 2), 303)]
    ret, layers, _ = c.compress_batch(["layerX.weight"] * 3, xs)
    assert ret == 0
    assert [L.step for L in layers] == [1, 2, 3]
    assert layers[1].type != "momentum_predicted" and layers[2].type != "momentum_predicted"


def test_shape_change_grouped_semantics_match_reference(product_lib, monkeypatch):
    """The grouped path groups by layer|dtype|shape: the reference gives
    steps 1, 1, 2 here (items 0 and 2 share a group)."""
    if not ob.have_ref():
        pytest.skip("reference build not present")
    grouped(monkeypatch)
    xs = [sincos((2, 2, 2, 2), 301), sincos((3, 2, 2, 2), 302), sincos((2, 2, 2, 2), 303)]
    ours = Codec(product_lib, client="client_0", param_count_threshold=THR)
    ours.lib.falcom_set_residual_codec(ours.h, b"raw")
    ref = Codec(ob.REF_SO, client="client_0", param_count_threshold=THR)
    _, A, _ = ours.compress_batch(["layerX.weight"] * 3, xs)
    _, B, _ = ref.compress_batch(["layerX.weight"] * 3, xs)
    assert [(a.type, a.step) for a in A] == [(b.type, b.step) for b in B]
    for a, b in zip(A, B):
        assert a.data == b.data
    assert ours.detailed_stats()[0]["step_count"] == ref.detailed_stats()[0]["step_count"]


def test_uint8_metadata_roundtrip(product_lib):
    c = Codec(product_lib, client="client_0", param_count_threshold=THR)
    x = ((401 + np.arange(8) * 7) & 0xFF).astype(np.uint8)
    L = c.compress_layer("metadata", x)
    assert L is not None and L.stored_dtype == "uint8" and L.codec == "zstd"
    y = c.decompress_layer(L, "metadata")
    assert y.dtype == np.uint8 and np.array_equal(x, y)


def test_sz3_memcpy_direct_decode_and_size_mismatch(product_lib):
    c = Codec(product_lib, client="client_0", param_count_threshold=1024 * 1024)
    vals = np.array([1.25, -2.5], np.float32)
    L = Layer(type="direct", codec="sz3_memcpy", data=vals.tobytes(), bitmap=b"", dominant_signs=b"",
              shape=(2,), original_dtype="float32", stored_dtype="float32", step=1,
              num_predicted_kernels=0, prediction_ratio=0, sign_mismatch_ratio=0, current_mean=0,
              current_std=0, prev_mean=0, prev_std=0, global_min=0, global_max=0)
    y = c.decompress_layer(L, "manual_sz3_memcpy")
    assert y is not None and np.array_equal(y, vals)
    L.data = np.float32(1.0).tobytes()
    assert c.decompress_layer(L, "bad_sz3_memcpy") is None     # NULL, never a zero array


def test_non_finite_inputs_do_not_crash(product_lib):
    c = Codec(product_lib, client="client_0", param_count_threshold=THR)
    x = np.array([0.0, -0.0, np.nan, np.inf, -np.inf, 1e-30, 1e30, -3.0], np.float32)
    L = c.compress_layer("nan_inf.weight", x)
    if L is not None:
        c.decompress_layer(L, "nan_inf.weight")


def test_grouped_failure_does_not_half_commit(product_lib, monkeypatch):
    grouped(monkeypatch)
    c = Codec(product_lib, client="client_0", param_count_threshold=THR)
    monkeypatch.setenv("FALCOM_FAULT_INJECT_COMPRESS_FAIL_AT", "1")
    ret, layers, errs = c.compress_batch(["faultA.weight", "faultB.weight"],
                                         [sincos((2, 2, 2, 2), 9), sincos((2, 2, 2, 2), 10)])
    monkeypatch.delenv("FALCOM_FAULT_INJECT_COMPRESS_FAIL_AT")
    assert ret != 0 and layers == [None, None]
    assert errs == [-2, -2]
    # nothing was committed: the next batch is still step 1
    ret, layers, _ = c.compress_batch(["faultA.weight", "faultB.weight"],
                                      [sincos((2, 2, 2, 2), 9), sincos((2, 2, 2, 2), 10)])
    assert ret == 0 and [L.step for L in layers] == [1, 1]


def test_stats_and_reset(product_lib):
    c = Codec(product_lib, client="c7", param_count_threshold=THR)
    for r in range(3):
        c.compress_batch(["a.weight", "b.bias"], [sincos((2, 2, 2, 2), r), sincos((8,), r)])
    s = c.stats()
    assert s["total_compressions"] == 6 and s["num_predictions"] == 2
    d = c.detailed_stats()
    assert d == [{"client_id": "c7", "history_length": 2, "step_count": 3, "num_memory_layers": 1}]
    c.lib.momentum_compressor_reset_client(c.h, b"c7")
    assert c.detailed_stats() == []
    _, L, _ = c.compress_batch(["a.weight"], [sincos((2, 2, 2, 2), 5)])
    assert L[0].step == 1


def test_model_container_roundtrip(product_lib):
    """MOMC container (reference :3600-3939) through compress_model /
    decompress_model."""
    from compressor_b200.abi import HostArray, NDArrayC, ndarray_to_numpy
    enc = Codec(product_lib, client="Client3", param_count_threshold=THR)
    dec = Codec(product_lib, client="Client3", param_count_threshold=THR)
    names = ["c1.weight", "c2.weight", "bn.bias"]
    for r in range(3):
        xs = [sincos((4, 2, 3, 3), r), sincos((8, 4, 1, 1), r + 5), sincos((16,), r + 9)]
        hs = [HostArray(x) for x in xs]
        grads = (ctypes.POINTER(NDArrayC) * 3)(*[ctypes.pointer(h.c) for h in hs])
        cn = (ctypes.c_char_p * 3)(*[n.encode() for n in names])
        size = ctypes.c_size_t(0)
        blob = enc.lib.momentum_compressor_compress_model(enc.h, grads, cn, 3, b"Client3", ctypes.byref(size))
        assert blob and size.value > 12
        raw = ctypes.string_at(blob, size.value)
        assert raw[:4] == (0x4D4F4D43).to_bytes(4, "little")
        buf = (ctypes.c_uint8 * len(raw)).from_buffer_copy(raw)
        names_out = ctypes.POINTER(ctypes.c_char_p)()
        nl = ctypes.c_size_t(0)
        arrs = dec.lib.momentum_compressor_decompress_model(dec.h, buf, len(raw), ctypes.byref(names_out),
                                                            ctypes.byref(nl))
        assert nl.value == 3
        for i in range(3):
            assert names_out[i].decode() == names[i]
            y = ndarray_to_numpy(arrs[i])
            assert y.shape == xs[i].shape and np.all(np.isfinite(y))
            if i == 2:
                assert np.array_equal(y, xs[i])      # lossless
            dec.lib.ndarray_destroy(arrs[i])


@pytest.mark.parametrize("prog", ["test_reference_state_oracle", "test_batch_state_equivalence",
                                  "test_runtime_contracts"])
def test_reference_c_programs_against_this_library(prog):
    exe = os.path.join(os.path.dirname(ob.REF_SO), "on_b200", prog)
    if not os.path.exists(exe):
        pytest.skip("reference C contract programs were not built against this library")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
    assert "ok - " in r.stdout

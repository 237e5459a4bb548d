"""Replay rounds on the CPU: the native writer and the host-mode loader
against an independent parser of the reference's layout
(profile_appfl_hot_rounds.py:47-72 read_round, benchmark_real.c:30-89), the
consistency checks, and error returns (NULL, as the reference loader)."""
import os
import struct

import numpy as np
import pytest

from compressor_b200 import replay

DTYPE_CODE = {np.dtype("float32"): 0, np.dtype("float64"): 1, np.dtype("int32"): 2,
              np.dtype("int64"): 3, np.dtype("uint8"): 4}
CODE_DTYPE = {v: k for k, v in DTYPE_CODE.items()}


def parse_round(path):
    """The layout, read field by field (little-endian)."""
    model = {}
    with open(path, "rb") as f:
        rnd = struct.unpack("<I", f.read(4))[0]
        client = f.read(64).split(b"\0", 1)[0].decode()
        count = struct.unpack("<Q", f.read(8))[0]
        for _ in range(count):
            name = f.read(256).split(b"\0", 1)[0].decode()
            shape8 = struct.unpack("<8Q", f.read(64))
            ndim = struct.unpack("<Q", f.read(8))[0]
            code = struct.unpack("<I", f.read(4))[0]
            size = struct.unpack("<Q", f.read(8))[0]
            raw = f.read(size)
            assert len(raw) == size
            model[name] = np.frombuffer(raw, dtype=CODE_DTYPE[code]).reshape(shape8[:ndim])
        assert f.read(1) == b""
    return rnd, client, model


def sample_tensors(seed=7):
    rng = np.random.default_rng(seed)
    return {
        "conv1.weight": rng.standard_normal((16, 3, 3, 3)).astype(np.float32),
        "layer1.0.conv1.weight": rng.standard_normal((32, 16, 1, 1)).astype(np.float32),
        "bn1.running_var": rng.random(16),                                   # float64
        "bn1.num_batches_tracked": np.array(1234567890123, dtype=np.int64),  # scalar
        "fc.bias": rng.integers(-5, 5, size=10).astype(np.int32),
        "mask": rng.integers(0, 255, size=33).astype(np.uint8),
        "empty": np.zeros((0, 4), dtype=np.float32),
    }


def write_raw(path, rnd, client, layers):
    """Hand-built file: layers = [(name, shape, ndim, code, size, payload)]."""
    with open(path, "wb") as f:
        f.write(struct.pack("<I", rnd))
        f.write(client.encode().ljust(64, b"\0"))
        f.write(struct.pack("<Q", len(layers)))
        for name, shape, ndim, code, size, payload in layers:
            f.write(name.encode().ljust(256, b"\0"))
            f.write(struct.pack("<8Q", *(list(shape) + [0] * (8 - len(shape)))))
            f.write(struct.pack("<Q", ndim))
            f.write(struct.pack("<I", code))
            f.write(struct.pack("<Q", size))
            f.write(payload)


def test_write_matches_reference_layout(tmp_path, product_lib):
    t = sample_tensors()
    p = str(tmp_path / "round3.bin")
    assert replay.write_round(p, 3, "Client7", t) == 0
    rnd, client, model = parse_round(p)
    assert (rnd, client) == (3, "Client7")
    assert list(model) == list(t)
    for k, v in t.items():
        assert model[k].dtype == v.dtype and model[k].shape == v.shape, k
        assert np.array_equal(model[k], v), k


def test_host_load_round_trip(tmp_path, product_lib):
    t = sample_tensors(11)
    p = str(tmp_path / "r.bin")
    assert replay.write_round(p, 9, "ClientA", t) == 0
    rnd, client, model, nbytes = replay.read_round(p)
    assert (rnd, client) == (9, "ClientA")
    assert nbytes == sum(v.nbytes for v in t.values())
    assert list(model) == list(t)
    for k, v in t.items():
        assert model[k].dtype == v.dtype and model[k].shape == v.shape, k
        assert np.array_equal(model[k], v), k
    with replay.ReplayRound(p, "host") as r:
        assert r.n == len(t)
        # items are ready for compress_batch: names and gradients set
        for i, k in enumerate(t):
            it = r.items[i]
            assert it.layer_name.decode() == k
            assert not it.compressed and it.error == 0
            assert it.gradient.contents.total_size == t[k].size
            assert it.gradient.contents.ndim == t[k].ndim
            assert r.ptrs[i] % 256 == 0


def test_hand_built_file_reads(tmp_path, product_lib):
    """A file written by other tools (only the layout in common)."""
    a = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    p = str(tmp_path / "hand.bin")
    write_raw(p, 1, "X" * 63, [("w", a.shape, 3, 0, a.nbytes, a.tobytes())])
    rnd, client, model, nbytes = replay.read_round(p)
    assert (rnd, client, nbytes) == (1, "X" * 63, a.nbytes)
    assert np.array_equal(model["w"], a)


@pytest.mark.parametrize("case", ["truncated_data", "bad_dtype", "size_mismatch", "ndim9",
                                  "short_header", "count_too_large"])
def test_inconsistent_files_are_refused(tmp_path, product_lib, case):
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    good = ("w", a.shape, 2, 0, a.nbytes, a.tobytes())
    p = str(tmp_path / f"{case}.bin")
    if case == "truncated_data":
        write_raw(p, 0, "c", [("w", a.shape, 2, 0, a.nbytes, a.tobytes()[:-4])])
    elif case == "bad_dtype":
        write_raw(p, 0, "c", [("w", a.shape, 2, 9, a.nbytes, a.tobytes())])
    elif case == "size_mismatch":
        write_raw(p, 0, "c", [("w", a.shape, 2, 0, a.nbytes - 4, a.tobytes()[:-4])])
    elif case == "ndim9":
        write_raw(p, 0, "c", [good])
        raw = bytearray(open(p, "rb").read())
        struct.pack_into("<Q", raw, 76 + 256 + 64, 9)
        open(p, "wb").write(bytes(raw))
    elif case == "short_header":
        open(p, "wb").write(b"\x01\x00\x00")
    elif case == "count_too_large":
        write_raw(p, 0, "c", [good])
        raw = bytearray(open(p, "rb").read())
        struct.pack_into("<Q", raw, 68, 1 << 40)
        open(p, "wb").write(bytes(raw))
    with pytest.raises(OSError):
        replay.ReplayRound(p, "host")


def test_missing_file(tmp_path, product_lib):
    with pytest.raises(OSError):
        replay.ReplayRound(str(tmp_path / "nope.bin"), "host")


def test_writer_rejects_bad_items(tmp_path, product_lib):
    with pytest.raises(TypeError):
        replay.write_round(str(tmp_path / "x.bin"), 0, "c", {"a": np.zeros(3, dtype=np.float16)})
    assert replay.write_round(str(tmp_path / "x.bin"), 0, "c", {"n" * 300: np.zeros(3, np.float32)}) != 0

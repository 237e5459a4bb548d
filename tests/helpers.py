"""Shared helpers of the parity tests."""
from __future__ import annotations

import numpy as np

from oracle import binding as ob


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(a), 1e-30))


def frame_content(frame: bytes) -> bytes:
    return ob.zstd_decompress(frame) if frame else b""


def residual_floats(layer) -> np.ndarray:
    """Residual / direct payload as float32 for raw ("sz3_memcpy") layers."""
    assert layer.codec == "sz3_memcpy", layer.codec
    return np.frombuffer(layer.data, np.float32)


def decode_codes(layer, n: int):
    """(scale, int8 codes) of a q8 / int4 payload."""
    scale = np.frombuffer(layer.data[:4], np.float32)[0]
    if layer.codec == "q8":
        return scale, np.frombuffer(layer.data[4:4 + n], np.int8)
    assert layer.codec == "int4"
    return scale, ob.unpack_int4(np.frombuffer(layer.data[4:], np.uint8), n)


def seeded(shape, seed, scale=1e-3, zeros_every=0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(shape) * scale).astype(np.float32)
    if zeros_every:
        x.reshape(-1)[::zeros_every] = 0.0
    return x

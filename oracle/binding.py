"""numpy front end of the CPU restatement oracle (oracle/falcom_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker; the product never imports it.

Also locates the reference build (oracle/_ref/libmomentum_compressor_ref.so),
which exports the same C ABI as the product library, and a libzstd handle for
decoding zstd frames in tests.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libfalcom_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmomentum_compressor_ref.so")


class Stats(ctypes.Structure):
    _fields_ = [
        ("cur_mean", ctypes.c_float), ("cur_std", ctypes.c_float),
        ("prev_mean", ctypes.c_float), ("prev_std", ctypes.c_float),
        ("gmin", ctypes.c_float), ("gmax", ctypes.c_float),
        ("predicted", ctypes.c_int64), ("mismatches", ctypes.c_int64),
        ("predicted_elems", ctypes.c_int64),
        ("prediction_ratio", ctypes.c_float), ("sign_mismatch_ratio", ctypes.c_float),
    ]


_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
        i64 = ctypes.c_int64
        L.fo_triple_stats.argtypes = [f32p, f32p, i64, ctypes.POINTER(Stats)]
        L.fo_sign_consistency.argtypes = [f32p, i64, i64, ctypes.c_float, u8p, i8p]
        L.fo_sign_consistency.restype = i64
        L.fo_encode_momentum.argtypes = [f32p, f32p, f32p, i64, i64, i64, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_float, f32p, u8p, u8p,
                                         ctypes.POINTER(Stats)]
        L.fo_encode_momentum.restype = i64
        L.fo_decode_momentum.argtypes = [f32p, ctypes.c_void_p, i64, ctypes.c_void_p, i64,
                                         ctypes.c_void_p, f32p, i64, i64, i64,
                                         ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_float, ctypes.c_float, f32p]
        L.fo_decode_momentum.restype = ctypes.c_int
        L.fo_quantize.argtypes = [f32p, i64, ctypes.c_int, i8p]
        L.fo_quantize.restype = ctypes.c_float
        L.fo_dequantize.argtypes = [i8p, i64, ctypes.c_float, f32p]
        L.fo_pack_int4.argtypes = [i8p, i64, u8p]
        L.fo_unpack_int4.argtypes = [u8p, i64, i8p]
        L.fo_pack_bits.argtypes = [u8p, i64, u8p]
        _lib = L
    return _lib


def stats_dict(st: Stats) -> dict:
    return {k: getattr(st, k) for k, _ in Stats._fields_}


def encode_momentum(cur: np.ndarray, prev: np.ndarray, mem: np.ndarray, step: int = 2,
                    lr: float = 0.07, threshold: float = 0.5):
    """One encoder step on a 4-D layer; mem is updated in place.
    Returns dict(residual, bitmap, signs, stats)."""
    assert cur.ndim == 4 and cur.dtype == np.float32
    oc, ic, h, w = cur.shape
    K, ks = oc * ic, h * w
    cur = np.ascontiguousarray(cur).reshape(-1)
    prev = np.ascontiguousarray(prev, dtype=np.float32).reshape(-1)
    assert mem.dtype == np.float32 and mem.flags.c_contiguous
    res = np.empty_like(cur)
    bitmap = np.zeros((K + 7) // 8, np.uint8)
    signs = np.zeros(max((K + 7) // 8, 1), np.uint8)
    st = Stats()
    nsb = lib().fo_encode_momentum(cur, prev, mem.reshape(-1), oc, ic, ks, step, lr, threshold,
                                   res, bitmap, signs, ctypes.byref(st))
    return {"residual": res, "bitmap": bitmap, "signs": signs[:nsb].copy(), "stats": stats_dict(st)}


def decode_momentum(residual: np.ndarray, bitmap: Optional[bytes], signs: Optional[bytes],
                    prev_dec: Optional[np.ndarray], mem: np.ndarray, shape,
                    cur_mean, cur_std, prev_mean, prev_std, lr: float = 0.07):
    """Returns (recon, appended_to_history: bool); mem updated in place."""
    oc, ic, h, w = shape
    residual = np.ascontiguousarray(residual, dtype=np.float32).reshape(-1)
    recon = np.empty_like(residual)
    bm = np.frombuffer(bitmap, np.uint8) if bitmap else None
    sg = np.frombuffer(signs, np.uint8) if signs else None
    pv = np.ascontiguousarray(prev_dec, dtype=np.float32).reshape(-1) if prev_dec is not None else None
    rc = lib().fo_decode_momentum(
        residual, bm.ctypes.data if bm is not None else None, 0 if bm is None else bm.size,
        sg.ctypes.data if sg is not None else None, 0 if sg is None else sg.size,
        pv.ctypes.data if pv is not None else None, mem.reshape(-1), oc, ic, h * w,
        cur_mean, cur_std, prev_mean, prev_std, lr, recon)
    return recon.reshape(shape), rc == 0


def quantize(x: np.ndarray, qmax: int):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    codes = np.empty(x.size, np.int8)
    scale = lib().fo_quantize(x, x.size, qmax, codes)
    return np.float32(scale), codes


def dequantize(codes: np.ndarray, scale: float) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    out = np.empty(codes.size, np.float32)
    lib().fo_dequantize(codes, codes.size, scale, out)
    return out


def pack_int4(codes: np.ndarray) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    out = np.zeros((codes.size + 1) // 2, np.uint8)
    lib().fo_pack_int4(codes, codes.size, out)
    return out


def unpack_int4(packed: np.ndarray, n: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.empty(n, np.int8)
    lib().fo_unpack_int4(packed, n, out)
    return out


# ---------------------------------------------------------------- libzstd
_zstd = None


def zstd():
    global _zstd
    if _zstd is None:
        z = ctypes.CDLL("libzstd.so.1")
        z.ZSTD_getFrameContentSize.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        z.ZSTD_getFrameContentSize.restype = ctypes.c_ulonglong
        z.ZSTD_decompress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
        z.ZSTD_decompress.restype = ctypes.c_size_t
        z.ZSTD_compress.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        z.ZSTD_compress.restype = ctypes.c_size_t
        z.ZSTD_compressBound.argtypes = [ctypes.c_size_t]
        z.ZSTD_compressBound.restype = ctypes.c_size_t
        z.ZSTD_isError.argtypes = [ctypes.c_size_t]
        z.ZSTD_isError.restype = ctypes.c_uint
        _zstd = z
    return _zstd


def zstd_decompress(frame: bytes) -> bytes:
    z = zstd()
    src = ctypes.create_string_buffer(frame, len(frame))
    n = z.ZSTD_getFrameContentSize(src, len(frame))
    if n >= (1 << 63):
        raise ValueError("zstd frame without content size")
    dst = ctypes.create_string_buffer(max(int(n), 1))
    rc = z.ZSTD_decompress(dst, int(n), src, len(frame))
    if z.ZSTD_isError(rc):
        raise ValueError("zstd decompression failed")
    return dst.raw[:rc]


def zstd_compress(data: bytes, level: int = 10) -> bytes:
    z = zstd()
    cap = z.ZSTD_compressBound(len(data))
    dst = ctypes.create_string_buffer(cap)
    rc = z.ZSTD_compress(dst, cap, data, len(data), level)
    if z.ZSTD_isError(rc):
        raise ValueError("zstd compression failed")
    return dst.raw[:rc]


def have_ref() -> bool:
    return os.path.exists(REF_SO)

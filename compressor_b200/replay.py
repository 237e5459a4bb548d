"""Replay rounds: captured client updates stored one round per file.

The layout is the one the reference's replay tools read
(benchmark_real.c:30-89 ``load_test_data``;
cuda_feasibility/profile_appfl_hot_rounds.py:47-72 ``read_round``)::

    u32 round | char client_id[64] | u64 layer_count
    per layer: char name[256] | u64 shape[8] | u64 ndim | u32 dtype |
               u64 data_size | data_size bytes          (little-endian)

Reading and writing go through the library's native loader
(``falcom_replay_*``): a round is read into one host block, or streamed
through pinned staging buffers into one device block, and comes back as the
BatchItem array ``momentum_compressor_compress_batch`` takes.
"""
from __future__ import annotations

import ctypes
import os
from collections import OrderedDict
from typing import Dict, Tuple

import numpy as np

from .abi import DTYPE_TO_NP, NP_TO_DTYPE, BatchItemC, NDArrayC, bind_replay

LOC_HOST, LOC_DEVICE = 1, 2


def _lib(lib_path: str = None) -> ctypes.CDLL:
    if lib_path is None:
        from . import build
        lib_path = build.OUT
    lib = ctypes.CDLL(os.path.abspath(lib_path))
    bind_replay(lib)
    return lib


class ReplayRound:
    """One replay round loaded by the native loader.

    ``items`` / ``n`` feed ``momentum_compressor_compress_batch`` directly;
    ``names``, ``shapes``, ``dtypes``, ``round``, ``client`` and ``nbytes``
    (the reference's ``original_bytes``) describe it.  The tensors stay valid
    until ``close()``."""

    def __init__(self, path: str, location: str = "device", device: int = 0, lib_path: str = None):
        self.lib = _lib(lib_path)
        loc = {"host": LOC_HOST, "device": LOC_DEVICE}[location]
        self.location = location
        self.h = self.lib.falcom_replay_open(os.fsencode(path), loc, device)
        if not self.h:
            raise OSError(f"cannot read replay round {path}")
        self.n = int(self.lib.falcom_replay_count(self.h))
        self.round = int(self.lib.falcom_replay_round(self.h))
        self.client = self.lib.falcom_replay_client(self.h).decode("utf-8", errors="replace")
        self.nbytes = int(self.lib.falcom_replay_bytes(self.h))
        self.items = self.lib.falcom_replay_items(self.h)
        self.names, self.shapes, self.dtypes, self.ptrs = [], [], [], []
        for i in range(self.n):
            it = self.items[i]
            a = it.gradient.contents
            self.names.append(it.layer_name.decode("utf-8", errors="replace"))
            self.shapes.append(tuple(int(a.shape[d]) for d in range(a.ndim)))
            self.dtypes.append(DTYPE_TO_NP[a.dtype])
            self.ptrs.append(int(a.data))

    def numpy(self, i: int) -> np.ndarray:
        """Host copy of tensor i (host-resident rounds only)."""
        if self.location != "host":
            raise ValueError("numpy() reads host-resident rounds; use the device pointers in .ptrs")
        dt = self.dtypes[i]
        n = int(np.prod(self.shapes[i])) if self.shapes[i] else 1
        buf = ctypes.string_at(self.ptrs[i], n * dt.itemsize)
        return np.frombuffer(buf, dtype=dt).reshape(self.shapes[i]).copy()

    def close(self) -> None:
        if self.h:
            self.lib.falcom_replay_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def read_round(path: str, location: str = "host", device: int = 0,
               lib_path: str = None) -> Tuple[int, str, "OrderedDict[str, np.ndarray]", int]:
    """(round, client_id, name -> array, original_bytes), as the reference's
    ``read_round`` returns; arrays are host numpy copies."""
    with ReplayRound(path, "host", device, lib_path) as r:
        model = OrderedDict((r.names[i], r.numpy(i)) for i in range(r.n))
        return r.round, r.client, model, r.nbytes


def write_round(path: str, round_idx: int, client_id: str, tensors: Dict[str, np.ndarray],
                lib_path: str = None) -> int:
    """Writes host arrays as one replay round; returns 0 or a negative
    ErrorCode."""
    lib = _lib(lib_path)
    names = list(tensors)
    arrs = []
    for k in names:
        a = np.asarray(tensors[k])
        if a.dtype not in NP_TO_DTYPE:
            raise TypeError(f"unsupported dtype {a.dtype}")
        arrs.append(a if a.flags.c_contiguous else a.copy())   # keeps 0-d scalars 0-d
    keep = [k.encode() for k in names]
    shapes = [(ctypes.c_size_t * max(1, a.ndim))(*a.shape) for a in arrs]
    cs = []
    for a, sh in zip(arrs, shapes):
        c = NDArrayC()
        c.data = a.ctypes.data
        c.shape = sh
        c.ndim = a.ndim
        c.total_size = a.size
        c.dtype = NP_TO_DTYPE[a.dtype]
        cs.append(c)
    items = (BatchItemC * max(1, len(names)))()
    for i, c in enumerate(cs):
        items[i].layer_name = keep[i]
        items[i].gradient = ctypes.pointer(c)
    return int(lib.falcom_replay_write(os.fsencode(path), int(round_idx), client_id.encode(), items, len(names)))

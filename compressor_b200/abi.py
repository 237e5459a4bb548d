"""ctypes mirror of the momentum_compressor.h C ABI.

The struct layouts are the frozen ones of the reference interface
(Gonglz/Compressor momentum_compressor.h:84-152, mirrored by
EB-FaLCom/src/appfl/compressor/FalComC.py:47-105).  ``Codec`` wraps any shared
library that exports that ABI: this package's ``libmomentum_compressor.so`` or
a reference build of the same interface.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

MAX_NDIM = 8

DTYPE_FLOAT32, DTYPE_FLOAT64, DTYPE_INT32, DTYPE_INT64, DTYPE_UINT8, DTYPE_UNKNOWN = range(6)
NP_TO_DTYPE = {
    np.dtype("float32"): DTYPE_FLOAT32,
    np.dtype("float64"): DTYPE_FLOAT64,
    np.dtype("int32"): DTYPE_INT32,
    np.dtype("int64"): DTYPE_INT64,
    np.dtype("uint8"): DTYPE_UINT8,
}
DTYPE_TO_NP = {v: k for k, v in NP_TO_DTYPE.items()}

ERROR_NONE = 0
ERROR_ALLOCATION = -1
ERROR_COMPRESSION = -2
ERROR_DECOMPRESSION = -3
ERROR_INVALID_PARAM = -4


class NDArrayC(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("shape", ctypes.POINTER(ctypes.c_size_t)),
        ("ndim", ctypes.c_size_t),
        ("total_size", ctypes.c_size_t),
        ("dtype", ctypes.c_int),
    ]


class CompressorConfigC(ctypes.Structure):
    _fields_ = [
        ("momentum_lr", ctypes.c_float),
        ("consistency_threshold", ctypes.c_float),
        ("lossless_compressor", ctypes.c_char * 32),
        ("error_bounding_mode", ctypes.c_char * 16),
        ("error_bound", ctypes.c_float),
        ("sz3_lib_path", ctypes.c_char * 512),
        ("param_count_threshold", ctypes.c_size_t),
        ("max_history_length", ctypes.c_int),
    ]


class CompressedLayerDataC(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_char * 32),
        ("codec", ctypes.c_char * 16),
        ("data", ctypes.POINTER(ctypes.c_uint8)),
        ("data_size", ctypes.c_size_t),
        ("bitmap", ctypes.POINTER(ctypes.c_uint8)),
        ("bitmap_size", ctypes.c_size_t),
        ("dominant_signs", ctypes.POINTER(ctypes.c_uint8)),
        ("dominant_signs_size", ctypes.c_size_t),
        ("shape", ctypes.c_size_t * MAX_NDIM),
        ("ndim", ctypes.c_size_t),
        ("original_dtype", ctypes.c_char * 16),
        ("stored_dtype", ctypes.c_char * 16),
        ("step", ctypes.c_int),
        ("num_predicted_kernels", ctypes.c_int),
        ("prediction_ratio", ctypes.c_float),
        ("sign_mismatch_ratio", ctypes.c_float),
        ("current_mean", ctypes.c_float),
        ("current_std", ctypes.c_float),
        ("prev_mean", ctypes.c_float),
        ("prev_std", ctypes.c_float),
        ("global_min", ctypes.c_float),
        ("global_max", ctypes.c_float),
        ("breakdown_stats_time", ctypes.c_double),
        ("breakdown_normalize_time", ctypes.c_double),
        ("breakdown_consistency_time", ctypes.c_double),
        ("breakdown_prediction_time", ctypes.c_double),
        ("breakdown_residual_compress_time", ctypes.c_double),
        ("breakdown_bitmap_compress_time", ctypes.c_double),
        ("breakdown_metadata_time", ctypes.c_double),
        ("breakdown_total_time", ctypes.c_double),
    ]


class BatchItemC(ctypes.Structure):
    _fields_ = [
        ("layer_name", ctypes.c_char_p),
        ("gradient", ctypes.POINTER(NDArrayC)),
        ("compressed", ctypes.POINTER(CompressedLayerDataC)),
        ("error", ctypes.c_int),
    ]


class CompressionStatsC(ctypes.Structure):
    _fields_ = [
        ("total_compressions", ctypes.c_size_t),
        ("avg_prediction_ratio", ctypes.c_float),
        ("std_prediction_ratio", ctypes.c_float),
        ("avg_sign_mismatch_ratio", ctypes.c_float),
        ("num_predictions", ctypes.c_size_t),
    ]


class ClientStatsC(ctypes.Structure):
    _fields_ = [
        ("client_id", ctypes.c_char * 256),
        ("history_length", ctypes.c_size_t),
        ("step_count", ctypes.c_int),
        ("num_memory_layers", ctypes.c_size_t),
    ]


class DetailedStatsC(ctypes.Structure):
    _fields_ = [
        ("compression", CompressionStatsC),
        ("clients", ctypes.POINTER(ClientStatsC)),
        ("num_clients", ctypes.c_size_t),
    ]


# Every entry point of the reference header (momentum_compressor.h:169-460)
# plus momentum_compressor_get_last_breakdown (defined at
# momentum_compressor_openmp_simd_final.c:197).
ABI_SYMBOLS = (
    "momentum_compressor_create", "momentum_compressor_destroy",
    "momentum_compressor_set_client", "momentum_compressor_compress_layer",
    "momentum_compressor_decompress_layer", "momentum_compressor_compress_batch",
    "momentum_compressor_decompress_batch", "momentum_compressor_reset_client",
    "momentum_compressor_reset_all", "momentum_compressor_print_stats",
    "momentum_compressor_get_stats", "momentum_compressor_get_detailed_stats",
    "compression_stats_free", "detailed_stats_free",
    "momentum_compressor_set_log_level", "momentum_compressor_set_client_context",
    "momentum_compressor_get_log_level", "momentum_compressor_get_current_client_id",
    "momentum_compressor_compress_model", "momentum_compressor_decompress_model",
    "ndarray_create", "ndarray_destroy", "ndarray_copy", "compressed_layer_data_free",
    "momentum_compressor_default_config", "momentum_compressor_enable_breakdown",
    "momentum_compressor_print_breakdown", "momentum_compressor_get_last_breakdown",
)


def _bind(lib: ctypes.CDLL) -> None:
    P = ctypes.POINTER
    c_vp = ctypes.c_void_p
    sigs = {
        "momentum_compressor_create": ([P(CompressorConfigC)], c_vp),
        "momentum_compressor_destroy": ([c_vp], None),
        "momentum_compressor_set_client": ([c_vp, ctypes.c_char_p], None),
        "momentum_compressor_compress_layer": ([c_vp, ctypes.c_char_p, P(NDArrayC)], P(CompressedLayerDataC)),
        "momentum_compressor_decompress_layer": (
            [c_vp, P(CompressedLayerDataC), ctypes.c_char_p, ctypes.c_char_p], P(NDArrayC)),
        "momentum_compressor_compress_batch": ([c_vp, P(BatchItemC), ctypes.c_size_t, ctypes.c_char_p], ctypes.c_int),
        "momentum_compressor_decompress_batch": (
            [c_vp, P(BatchItemC), ctypes.c_size_t, ctypes.c_char_p, P(P(NDArrayC))], ctypes.c_int),
        "momentum_compressor_reset_client": ([c_vp, ctypes.c_char_p], None),
        "momentum_compressor_reset_all": ([c_vp], None),
        "momentum_compressor_print_stats": ([c_vp], None),
        "momentum_compressor_get_stats": ([c_vp], P(CompressionStatsC)),
        "momentum_compressor_get_detailed_stats": ([c_vp], P(DetailedStatsC)),
        "compression_stats_free": ([P(CompressionStatsC)], None),
        "detailed_stats_free": ([P(DetailedStatsC)], None),
        "momentum_compressor_set_log_level": ([c_vp, ctypes.c_char_p], None),
        "momentum_compressor_set_client_context": ([c_vp, ctypes.c_char_p], None),
        "momentum_compressor_get_log_level": ([c_vp], ctypes.c_int),
        "momentum_compressor_get_current_client_id": ([c_vp], ctypes.c_char_p),
        "momentum_compressor_compress_model": (
            [c_vp, P(P(NDArrayC)), P(ctypes.c_char_p), ctypes.c_size_t, ctypes.c_char_p,
             P(ctypes.c_size_t)], P(ctypes.c_uint8)),
        "momentum_compressor_decompress_model": (
            [c_vp, P(ctypes.c_uint8), ctypes.c_size_t, P(P(ctypes.c_char_p)), P(ctypes.c_size_t)],
            P(P(NDArrayC))),
        "ndarray_create": ([P(ctypes.c_size_t), ctypes.c_size_t, ctypes.c_int], P(NDArrayC)),
        "ndarray_destroy": ([P(NDArrayC)], None),
        "ndarray_copy": ([P(NDArrayC)], P(NDArrayC)),
        "compressed_layer_data_free": ([P(CompressedLayerDataC)], None),
        "momentum_compressor_default_config": ([], CompressorConfigC),
        "momentum_compressor_enable_breakdown": ([ctypes.c_int], None),
        "momentum_compressor_print_breakdown": ([], None),
    }
    for name, (argt, rest) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = argt
        fn.restype = rest


def cstr(raw: bytes) -> str:
    return bytes(raw).split(b"\0", 1)[0].decode("utf-8", errors="replace")


@dataclass
class Layer:
    """Python-owned copy of one CompressedLayerData."""
    type: str
    codec: str
    data: bytes
    bitmap: bytes
    dominant_signs: bytes
    shape: tuple
    original_dtype: str
    stored_dtype: str
    step: int
    num_predicted_kernels: int
    prediction_ratio: float
    sign_mismatch_ratio: float
    current_mean: float
    current_std: float
    prev_mean: float
    prev_std: float
    global_min: float
    global_max: float
    extra: dict = field(default_factory=dict)

    @staticmethod
    def from_c(c: CompressedLayerDataC, copy_payload: bool = True) -> "Layer":
        def grab(ptr, size):
            if not copy_payload or not ptr or size == 0:
                return b""
            return ctypes.string_at(ptr, size)
        return Layer(
            type=cstr(c.type), codec=cstr(c.codec),
            data=grab(c.data, c.data_size), bitmap=grab(c.bitmap, c.bitmap_size),
            dominant_signs=grab(c.dominant_signs, c.dominant_signs_size),
            shape=tuple(int(c.shape[i]) for i in range(c.ndim)),
            original_dtype=cstr(c.original_dtype), stored_dtype=cstr(c.stored_dtype),
            step=int(c.step), num_predicted_kernels=int(c.num_predicted_kernels),
            prediction_ratio=float(c.prediction_ratio), sign_mismatch_ratio=float(c.sign_mismatch_ratio),
            current_mean=float(c.current_mean), current_std=float(c.current_std),
            prev_mean=float(c.prev_mean), prev_std=float(c.prev_std),
            global_min=float(c.global_min), global_max=float(c.global_max),
            extra={"data_size": int(c.data_size), "bitmap_size": int(c.bitmap_size),
                   "dominant_signs_size": int(c.dominant_signs_size)},
        )

    def to_c(self):
        """Build a CompressedLayerDataC pointing at Python-owned buffers.
        Returns (struct, keepalive)."""
        c = CompressedLayerDataC()
        c.type = self.type.encode()
        c.codec = self.codec.encode()
        c.original_dtype = self.original_dtype.encode()
        c.stored_dtype = self.stored_dtype.encode()
        keep = []
        for name in ("data", "bitmap", "dominant_signs"):
            blob = getattr(self, name)
            if blob:
                buf = (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)
                keep.append(buf)
                setattr(c, name, ctypes.cast(buf, ctypes.POINTER(ctypes.c_uint8)))
                setattr(c, name + "_size", len(blob))
        for i, d in enumerate(self.shape):
            c.shape[i] = int(d)
        c.ndim = len(self.shape)
        c.step = self.step
        c.num_predicted_kernels = self.num_predicted_kernels
        c.prediction_ratio = self.prediction_ratio
        c.sign_mismatch_ratio = self.sign_mismatch_ratio
        c.current_mean, c.current_std = self.current_mean, self.current_std
        c.prev_mean, c.prev_std = self.prev_mean, self.prev_std
        c.global_min, c.global_max = self.global_min, self.global_max
        return c, keep


class HostArray:
    """An NDArrayC that borrows a contiguous numpy array (kept alive here)."""

    def __init__(self, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        self.arr = arr
        self.shape_buf = (ctypes.c_size_t * arr.ndim)(*arr.shape)
        self.c = NDArrayC()
        self.c.data = arr.ctypes.data
        self.c.shape = self.shape_buf
        self.c.ndim = arr.ndim
        self.c.total_size = arr.size
        self.c.dtype = NP_TO_DTYPE[arr.dtype]


class DeviceArray:
    """An NDArrayC that borrows device memory given as an integer address."""

    def __init__(self, ptr: int, shape: Sequence[int], dtype=np.float32):
        self.shape_buf = (ctypes.c_size_t * len(shape))(*shape)
        self.c = NDArrayC()
        self.c.data = int(ptr)
        self.c.shape = self.shape_buf
        self.c.ndim = len(shape)
        self.c.total_size = int(np.prod(shape))
        self.c.dtype = NP_TO_DTYPE[np.dtype(dtype)]


def ndarray_to_numpy(p) -> np.ndarray:
    a = p.contents
    dt = DTYPE_TO_NP[a.dtype]
    shape = tuple(a.shape[i] for i in range(a.ndim))
    nbytes = a.total_size * dt.itemsize
    buf = ctypes.string_at(a.data, nbytes)
    return np.frombuffer(buf, dtype=dt).reshape(shape).copy()


class Codec:
    """One MomentumCompressor instance of a library exporting the ABI."""

    def __init__(self, lib_path: str, client: str = "Client1", **cfg):
        self.lib = ctypes.CDLL(os.path.abspath(lib_path))
        _bind(self.lib)
        if hasattr(self.lib, "falcom_set_residual_codec"):
            bind_extensions(self.lib)
        c = self.lib.momentum_compressor_default_config()
        for k, v in cfg.items():
            if isinstance(v, str):
                v = v.encode()
            setattr(c, k, v)
        self.config = c
        self.h = self.lib.momentum_compressor_create(ctypes.byref(c))
        if not self.h:
            raise RuntimeError("momentum_compressor_create failed")
        self.client = client
        self.lib.momentum_compressor_set_client(self.h, client.encode())

    def close(self):
        if self.h:
            self.lib.momentum_compressor_destroy(self.h)
            self.h = None

    # -- state checkpoint (extension) ---------------------------------------
    def save_state(self, path: str) -> int:
        return self.lib.falcom_state_save(self.h, os.fsencode(path))

    def load_state(self, path: str) -> int:
        return self.lib.falcom_state_load(self.h, os.fsencode(path))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- batch API ---------------------------------------------------------
    def compress_batch_raw(self, names: List[str], arrays: List, client: Optional[str] = None):
        """arrays: HostArray / DeviceArray.  Returns (ret, items) with the C
        items still owning their CompressedLayerData."""
        n = len(names)
        items = (BatchItemC * n)()
        self._keep_names = [nm.encode() for nm in names]
        for i in range(n):
            items[i].layer_name = self._keep_names[i]
            items[i].gradient = ctypes.pointer(arrays[i].c)
        ret = self.lib.momentum_compressor_compress_batch(
            self.h, items, n, (client or self.client).encode())
        return ret, items

    def free_items(self, items):
        for it in items:
            if it.compressed:
                self.lib.compressed_layer_data_free(it.compressed)
                it.compressed = None

    def compress_batch(self, names: List[str], arrays: List[np.ndarray], client: Optional[str] = None):
        hs = [HostArray(a) for a in arrays]
        ret, items = self.compress_batch_raw(names, hs, client)
        layers = [Layer.from_c(it.compressed.contents) if it.compressed else None for it in items]
        errors = [int(it.error) for it in items]
        self.free_items(items)
        return ret, layers, errors

    def decompress_batch(self, names: List[str], layers: List[Layer], client: Optional[str] = None):
        n = len(names)
        items = (BatchItemC * n)()
        keep = []
        enc = [nm.encode() for nm in names]
        for i in range(n):
            items[i].layer_name = enc[i]
            if layers[i] is not None:
                c, k = layers[i].to_c()
                keep.append((c, k))
                items[i].compressed = ctypes.pointer(c)
        outs = (ctypes.POINTER(NDArrayC) * n)()
        ret = self.lib.momentum_compressor_decompress_batch(
            self.h, items, n, (client or self.client).encode(), outs)
        res = []
        for i in range(n):
            if outs[i]:
                res.append(ndarray_to_numpy(outs[i]))
                self.lib.ndarray_destroy(outs[i])
            else:
                res.append(None)
        return ret, res

    # -- per-layer API -----------------------------------------------------
    def compress_layer(self, name: str, arr: np.ndarray) -> Optional[Layer]:
        h = HostArray(arr)
        p = self.lib.momentum_compressor_compress_layer(self.h, name.encode(), ctypes.byref(h.c))
        if not p:
            return None
        layer = Layer.from_c(p.contents)
        self.lib.compressed_layer_data_free(p)
        return layer

    def decompress_layer(self, layer: Layer, name: str, client: Optional[str] = None):
        c, keep = layer.to_c()
        p = self.lib.momentum_compressor_decompress_layer(
            self.h, ctypes.byref(c), (client or self.client).encode(), name.encode())
        if not p:
            return None
        out = ndarray_to_numpy(p)
        self.lib.ndarray_destroy(p)
        return out

    def stats(self):
        p = self.lib.momentum_compressor_get_stats(self.h)
        s = p.contents
        d = {k: getattr(s, k) for k, _ in CompressionStatsC._fields_}
        self.lib.compression_stats_free(p)
        return d

    def detailed_stats(self):
        p = self.lib.momentum_compressor_get_detailed_stats(self.h)
        s = p.contents
        clients = [{"client_id": cstr(s.clients[i].client_id),
                    "history_length": s.clients[i].history_length,
                    "step_count": s.clients[i].step_count,
                    "num_memory_layers": s.clients[i].num_memory_layers}
                   for i in range(s.num_clients)]
        self.lib.detailed_stats_free(p)
        return clients


class PreparedBatch:
    """Reusable C-side batch for a fixed list of tensors: one BatchItem and one
    NDArray per tensor, built once; each round only the data pointers change.
    compress -> decompress -> release run without per-item Python work."""

    def __init__(self, lib: ctypes.CDLL, names: Sequence[str], shapes: Sequence[Sequence[int]],
                 dtype=np.float32):
        self.lib = lib
        self.n = len(names)
        self._names = [nm.encode() for nm in names]
        self._shapes = [(ctypes.c_size_t * len(s))(*s) for s in shapes]
        self.arrays = (NDArrayC * self.n)()
        self.items = (BatchItemC * self.n)()
        self.outs = (ctypes.POINTER(NDArrayC) * self.n)()
        code = NP_TO_DTYPE[np.dtype(dtype)]
        for i, s in enumerate(shapes):
            a = self.arrays[i]
            a.shape = self._shapes[i]
            a.ndim = len(s)
            a.total_size = int(np.prod(s))
            a.dtype = code
            self.items[i].layer_name = self._names[i]
            self.items[i].gradient = ctypes.pointer(a)
        lib.falcom_free_batch.argtypes = [ctypes.POINTER(BatchItemC), ctypes.c_size_t,
                                          ctypes.POINTER(ctypes.POINTER(NDArrayC))]
        lib.falcom_free_batch.restype = None

    def set_pointers(self, base: int, offsets_bytes: Sequence[int]) -> None:
        for i, o in enumerate(offsets_bytes):
            self.arrays[i].data = base + o

    def compress(self, handle, client: bytes) -> int:
        return self.lib.momentum_compressor_compress_batch(handle, self.items, self.n, client)

    def decompress(self, handle, client: bytes) -> int:
        return self.lib.momentum_compressor_decompress_batch(handle, self.items, self.n, client, self.outs)

    def payload_bytes(self) -> int:
        tot = 0
        for it in self.items:
            if it.compressed:
                c = it.compressed.contents
                tot += c.data_size + c.bitmap_size + c.dominant_signs_size
        return tot

    def release(self) -> None:
        self.lib.falcom_free_batch(self.items, self.n, self.outs)


def bind_extensions(lib: ctypes.CDLL) -> None:
    c_vp = ctypes.c_void_p
    lib.falcom_set_residual_codec.argtypes = [c_vp, ctypes.c_char_p]
    lib.falcom_set_frame_mode.argtypes = [c_vp, ctypes.c_char_p]
    lib.falcom_set_payload_location.argtypes = [c_vp, ctypes.c_int]
    lib.falcom_set_output_location.argtypes = [c_vp, ctypes.c_int]
    lib.falcom_set_stream.argtypes = [c_vp, c_vp]
    lib.falcom_last_error.argtypes = [c_vp]
    lib.falcom_last_error.restype = ctypes.c_char_p
    lib.falcom_last_launches.argtypes = [c_vp]
    lib.falcom_total_launches.argtypes = [c_vp]
    lib.falcom_total_launches.restype = ctypes.c_longlong
    lib.falcom_set_kernel_timing.argtypes = [c_vp, ctypes.c_int]
    lib.falcom_kernel_times.argtypes = [c_vp, ctypes.POINTER(ctypes.c_double),
                                        ctypes.POINTER(ctypes.c_longlong), ctypes.c_int]
    lib.falcom_kernel_name.argtypes = [ctypes.c_int]
    lib.falcom_kernel_name.restype = ctypes.c_char_p
    lib.falcom_set_aggregate.argtypes = [c_vp, c_vp, ctypes.POINTER(ctypes.c_size_t), ctypes.c_size_t,
                                         ctypes.c_float]
    lib.falcom_set_aggregate.restype = ctypes.c_int
    lib.falcom_set_aggregate_store.argtypes = [c_vp, ctypes.c_int]
    lib.falcom_set_aggregate_store.restype = ctypes.c_int
    lib.falcom_set_aggregate_only.argtypes = [c_vp, ctypes.c_int]
    lib.falcom_set_aggregate_only.restype = ctypes.c_int
    lib.falcom_set_aggregate_shards.argtypes = [c_vp, ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_int,
                                                ctypes.c_size_t]
    lib.falcom_set_aggregate_shards.restype = ctypes.c_int
    lib.falcom_shard_reduce.argtypes = [c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t,
                                        ctypes.POINTER(c_vp), c_vp]
    lib.falcom_shard_reduce.restype = ctypes.c_int
    lib.falcom_peer_allreduce.argtypes = [ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_int, ctypes.c_size_t,
                                          ctypes.c_size_t, c_vp]
    lib.falcom_peer_allreduce.restype = ctypes.c_int
    lib.falcom_peer_allreduce_sync.argtypes = [ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), ctypes.c_int,
                                               ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_uint32, c_vp]
    lib.falcom_peer_allreduce_sync.restype = ctypes.c_int
    lib.falcom_copy_sm.argtypes = [c_vp, c_vp, ctypes.c_size_t, ctypes.c_int, c_vp]
    lib.falcom_copy_sm.restype = ctypes.c_int
    lib.falcom_state_save.argtypes = [c_vp, ctypes.c_char_p]
    lib.falcom_state_save.restype = ctypes.c_int
    lib.falcom_state_load.argtypes = [c_vp, ctypes.c_char_p]
    lib.falcom_state_load.restype = ctypes.c_int
    bind_replay(lib)


def bind_replay(lib: ctypes.CDLL) -> None:
    """Replay-round entry points (falcom_replay_*); no instance needed."""
    c_vp = ctypes.c_void_p
    lib.falcom_replay_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int]
    lib.falcom_replay_open.restype = c_vp
    for name, rest in (("falcom_replay_count", ctypes.c_size_t), ("falcom_replay_round", ctypes.c_uint32),
                       ("falcom_replay_client", ctypes.c_char_p), ("falcom_replay_bytes", ctypes.c_size_t),
                       ("falcom_replay_items", ctypes.POINTER(BatchItemC)), ("falcom_replay_close", None)):
        fn = getattr(lib, name)
        fn.argtypes = [c_vp]
        fn.restype = rest
    lib.falcom_replay_write.argtypes = [ctypes.c_char_p, ctypes.c_uint32, ctypes.c_char_p,
                                        ctypes.POINTER(BatchItemC), ctypes.c_size_t]
    lib.falcom_replay_write.restype = ctypes.c_int


def kernel_times(lib: ctypes.CDLL, handle) -> dict:
    ms = (ctypes.c_double * 16)()
    cnt = (ctypes.c_longlong * 16)()
    k = lib.falcom_kernel_times(handle, ms, cnt, 16)
    return {lib.falcom_kernel_name(i).decode(): (ms[i], cnt[i]) for i in range(k)}

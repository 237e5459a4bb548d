"""Federated round over several GPUs: host-side plan of the server step.

Clients are independent units (the codec keys all encoder and decoder state
by client id, reference momentum_compressor_openmp_simd_final.c:452-471), so
they are block-distributed over the ranks, one process per GPU.  Each rank
compresses its clients' updates, decodes them on its server-side decoder
instance with the weighted aggregate fused into the decode
(``falcom_set_aggregate``), and one sum all-reduce of the flat aggregate over
NCCL finishes the global update.

Everything here but PeerAggregate is plain host logic (which clients a rank
owns, their weights, the aggregate layout and the collective); it runs the
same under the ``gloo`` backend on CPU tensors.  PeerAggregate maps the
aggregate buffers between the ranks' GPUs for the two NVLink peer-memory
sums (the reduce-scatter fused into the decoder, or the one-shot in-place
all-reduce kernel).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Sequence

import numpy as np


def shard(n_clients: int, world: int, rank: int) -> range:
    """Block distribution of client indices 0..n_clients-1 over `world`
    ranks: the first n_clients % world ranks get one extra client."""
    if world <= 0 or not 0 <= rank < world or n_clients < 0:
        raise ValueError(f"bad shard request: {n_clients} clients, rank {rank} of {world}")
    base, extra = divmod(n_clients, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def uniform_weights(n_clients: int) -> List[float]:
    """FedAvg weights of equally weighted clients."""
    if n_clients <= 0:
        raise ValueError("no clients")
    return [1.0 / n_clients] * n_clients


@dataclass
class AggregateLayout:
    """Flat float32 layout of one model update: element offset of every
    tensor, in state-dict order."""
    names: List[str]
    shapes: List[tuple]
    offsets: List[int]
    total: int

    @staticmethod
    def of(names: Sequence[str], shapes: Sequence[Sequence[int]], align: int = 1) -> "AggregateLayout":
        offs, o = [], 0
        for s in shapes:
            o = (o + align - 1) // align * align
            offs.append(o)
            o += int(np.prod(s))
        return AggregateLayout(list(names), [tuple(s) for s in shapes], offs, o)

    def c_offsets(self):
        return (ctypes.c_size_t * len(self.offsets))(*self.offsets)


def set_client_weight(lib, decoder_handle, aggregate_ptr: int, c_offsets, n: int, weight: float) -> None:
    """Points the decoder's fused aggregate at `aggregate_ptr` with the weight
    of the client whose batch it decodes next."""
    rc = lib.falcom_set_aggregate(decoder_handle, ctypes.c_void_p(aggregate_ptr), c_offsets, n, float(weight))
    if rc != 0:
        raise RuntimeError(f"falcom_set_aggregate failed ({rc}): {lib.falcom_last_error(decoder_handle)}")


def set_aggregate_store(lib, decoder_handle, store: bool) -> None:
    """Store mode of the decoder's fused aggregate: True for the first client
    of a round (the aggregate region is written, not read, so it needs no
    clearing), False for the clients that follow (added)."""
    rc = lib.falcom_set_aggregate_store(decoder_handle, 1 if store else 0)
    if rc != 0:
        raise RuntimeError(f"falcom_set_aggregate_store failed ({rc})")


def allreduce_aggregate(aggregate, dist=None, group=None) -> None:
    """Sum of the per-rank aggregates on every rank (no-op on one rank)."""
    if dist is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(aggregate, op=dist.ReduceOp.SUM, group=group)


def layer_chunks(numels: Sequence[int], n_chunks: int, fracs: Sequence[float] = None) -> List[tuple]:
    """Splits items 0..len(numels)-1, in order, into at most n_chunks
    contiguous runs [i0, i1) of about equal element counts, or of about the
    shares `fracs` of the elements (one per run, normalised; n_chunks is then
    len(fracs)): a run ends once the elements so far reach the share of the
    runs so far; every run holds at least one item."""
    n = len(numels)
    if n == 0:
        return []
    if fracs is not None:
        if len(fracs) == 0 or any(f <= 0 for f in fracs):
            raise ValueError("chunk shares must be positive")
        n_chunks = len(fracs)
    n_chunks = max(1, min(int(n_chunks), n))
    shares = [float(f) for f in fracs[:n_chunks]] if fracs is not None else [1.0] * n_chunks
    ends, c = [], 0.0
    for f in shares:
        c += f
        ends.append(c / sum(shares))
    total = float(sum(int(x) for x in numels))
    out, i0, acc = [], 0, 0
    for i, x in enumerate(numels):
        acc += int(x)
        left_items, left_chunks = n - (i + 1), n_chunks - len(out) - 1
        if left_chunks > 0 and (acc >= total * ends[len(out)] or left_items == left_chunks):
            out.append((i0, i + 1))
            i0 = i + 1
    out.append((i0, n))
    return out


class ChunkedAllreduce:
    """Sum all-reduce of the flat aggregate, one layer chunk at a time.

    The server step decodes the items of chunk 0, then chunk 1, ...; as soon
    as a chunk's decodes (with their fused aggregate additions) are queued,
    chunk_done(c) issues the all-reduce of that chunk's region of the
    aggregate as an asynchronous collective.  Under NCCL it runs on the
    process group's own stream, which waits only for the work already queued
    on the caller's stream, so it overlaps the codec work of the later
    chunks; wait() orders the caller's stream (or, under gloo, the host)
    after all of them.  Every rank issues the same chunks in the same order.
    No-op on one rank."""

    def __init__(self, aggregate, layout: AggregateLayout, chunks: Sequence[tuple], dist=None, group=None):
        self.aggregate = aggregate
        self.dist = dist
        self.group = group
        self.active = dist is not None and dist.is_initialized() and dist.get_world_size(group) > 1
        self.regions = []
        for i0, i1 in chunks:
            lo = layout.offsets[i0]
            last = i1 - 1
            hi = layout.offsets[last] + int(np.prod(layout.shapes[last]))
            self.regions.append((lo, hi))
        self.works = []

    def chunk_done(self, c: int) -> None:
        if not self.active:
            return
        lo, hi = self.regions[c]
        if hi > lo:
            self.works.append(self.dist.all_reduce(self.aggregate[lo:hi], op=self.dist.ReduceOp.SUM,
                                                   group=self.group, async_op=True))

    def wait(self) -> None:
        for w in self.works:
            w.wait()
        self.works = []


def shard_elems(total: int, nranks: int) -> int:
    """Elements per shard of a sharded aggregate: total / nranks rounded up
    to a multiple of 64, at least one tile (4096)."""
    if total < 0 or nranks < 1:
        raise ValueError("bad shard request")
    per = -(-total // nranks)
    return max(4096, -(-per // 64) * 64)


class PeerAggregate:
    """The server aggregate summed over the ranks' GPUs through NVLink peer
    memory, in one of two ways (`mode`):

    "fused": the sharded aggregate (falcom_set_aggregate_shards /
    falcom_shard_reduce).  The decodes of every rank's last client store into
    the owners' landing slots (the reduce-scatter fused into the decoder);
    `finish` then orders a barrier (a one-element all-reduce on the stream:
    every rank's decodes have landed), every rank's falcom_shard_reduce (its
    shard summed in rank order and stored into every rank's aggregate) and a
    second barrier.

    "oneshot": the decodes write local aggregates as without peers;
    `finish` orders a barrier, every rank's falcom_peer_allreduce (its shard
    loaded from every rank's aggregate, summed in rank order and stored back
    into every rank's aggregate: reduce-scatter and all-gather in one
    kernel, both directions of the links at once) and a second barrier.

    "synced": as "oneshot", with both barriers done inside the kernel
    (falcom_peer_allreduce_sync) over a block of flag words that follows
    each rank's aggregate in the same allocation; no NCCL call per round.
    `errors()` reads the rank's error word (a barrier wait that ran out).

    The buffers, on every rank: its aggregate and (fused) its landing buffer,
    nranks x shard floats each, zeroed, so padding between items stays 0,
    mapped into every other rank's address space over CUDA IPC.  After
    `finish` every rank's aggregate holds the global sum.  Every rank
    creates, uses and closes it at the same points, in the same mode."""

    MODES = ("fused", "oneshot", "synced")
    FLAG_BYTES = 256   # flag block behind a synced aggregate (18 words used)

    def __init__(self, torch, dist, total: int, device_index: int, mode: str = "fused"):
        from cuda.bindings import runtime as rt
        if mode not in self.MODES:
            raise ValueError(f"unknown peer aggregate mode {mode!r}")
        self.mode = mode
        self.rt, self.torch, self.dist = rt, torch, dist
        self._ok(rt.cudaSetDevice(int(device_index))[0], "cudaSetDevice")
        self.nranks = dist.get_world_size()
        self.rank = dist.get_rank()
        self.total = int(total)
        self.shard = shard_elems(self.total, self.nranks)
        nbytes = 4 * self.nranks * self.shard
        keys = ("agg", "land") if mode == "fused" else ("agg",)
        self.local = {}
        for key in keys:
            size = nbytes + (self.FLAG_BYTES if key == "agg" and mode == "synced" else 0)
            err, ptr = rt.cudaMalloc(size)
            self._ok(err, "cudaMalloc")
            self._ok(rt.cudaMemset(ptr, 0, size)[0], "cudaMemset")
            self.local[key] = int(ptr)
        self.epoch = 0
        self._ok(rt.cudaDeviceSynchronize()[0], "cudaDeviceSynchronize")
        mine = {}
        for key, ptr in self.local.items():
            err, h = rt.cudaIpcGetMemHandle(ptr)
            self._ok(err, "cudaIpcGetMemHandle")
            mine[key] = bytes(h.reserved)
        handles = [None] * self.nranks
        dist.all_gather_object(handles, mine)
        self.opened = []
        self.ptrs = {k: [0] * self.nranks for k in keys}
        failed = None
        for r in range(self.nranks):
            for key in keys:
                if r == self.rank:
                    self.ptrs[key][r] = self.local[key]
                    continue
                h = rt.cudaIpcMemHandle_t()
                h.reserved = handles[r][key]
                err, p = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
                if int(err) != 0:
                    failed = f"cudaIpcOpenMemHandle of rank {r}'s {key} failed ({err})"
                    continue
                self.ptrs[key][r] = int(p)
                self.opened.append(int(p))
        # every rank learns whether every rank mapped every peer buffer
        flag = torch.tensor([0 if failed else 1], dtype=torch.int32, device=torch.device("cuda", device_index))
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) != 1:
            self.close()
            raise RuntimeError(failed or "a peer could not map this rank's buffers")
        c_vp = ctypes.c_void_p
        self.c_land = (c_vp * self.nranks)(*self.ptrs["land"]) if mode == "fused" else None
        self.c_aggs = (c_vp * self.nranks)(*self.ptrs["agg"])
        # the flag blocks sit behind the nranks x shard floats of each aggregate
        self.c_flags = (c_vp * self.nranks)(*[p + nbytes for p in self.ptrs["agg"]]) if mode == "synced" else None
        self.flag_off = nbytes
        self.tiny = torch.zeros(1, device=torch.device("cuda", device_index))
        self.agg = torch.as_tensor(_DeviceFloats(self.local["agg"], self.total), device=self.tiny.device)

    @staticmethod
    def _ok(err, what):
        if int(err) != 0:
            raise RuntimeError(f"{what} failed ({err})")

    def enable(self, lib, decoder_handle) -> None:
        """Fused mode: the decoder's next decodes go to the owners' landing
        slots (no-op in oneshot mode)."""
        if self.mode != "fused":
            return
        rc = lib.falcom_set_aggregate_shards(decoder_handle, self.c_land, self.nranks, self.rank, self.shard)
        if rc != 0:
            raise RuntimeError(f"falcom_set_aggregate_shards failed ({rc})")

    def disable(self, lib, decoder_handle) -> None:
        if self.mode == "fused":
            lib.falcom_set_aggregate_shards(decoder_handle, None, 0, 0, 0)

    def finish(self, lib, stream_ptr: int) -> None:
        """After this rank's decodes are queued: barrier, the cross-rank sum
        (shard sum + all-gather, or the one-shot all-reduce), barrier (all on
        the current stream)."""
        if self.mode == "synced":
            self.epoch = (self.epoch + 1) & 0xFFFFFFFF
            rc = lib.falcom_peer_allreduce_sync(self.c_aggs, self.c_flags, self.nranks, self.rank, self.shard,
                                                self.total, self.epoch, ctypes.c_void_p(stream_ptr))
            if rc != 0:
                raise RuntimeError(f"falcom_peer_allreduce_sync failed ({rc})")
            return
        self.dist.all_reduce(self.tiny)
        if self.mode == "fused":
            rc = lib.falcom_shard_reduce(ctypes.c_void_p(self.local["land"]), self.nranks, self.rank, self.shard,
                                         self.total, self.c_aggs, ctypes.c_void_p(stream_ptr))
            what = "falcom_shard_reduce"
        else:
            rc = lib.falcom_peer_allreduce(self.c_aggs, self.nranks, self.rank, self.shard, self.total,
                                           ctypes.c_void_p(stream_ptr))
            what = "falcom_peer_allreduce"
        if rc != 0:
            raise RuntimeError(f"{what} failed ({rc})")
        self.dist.all_reduce(self.tiny)

    def errors(self) -> int:
        """Synced mode: this rank's error word (nonzero once a barrier wait in
        the kernel ran out); 0 in the other modes.  Synchronises the device."""
        if self.mode != "synced":
            return 0
        self.torch.cuda.synchronize()
        buf = (ctypes.c_uint32 * 1)()
        err = self.rt.cudaMemcpy(ctypes.addressof(buf), self.local["agg"] + self.flag_off + 4 * 17, 4,
                                 self.rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)[0]
        self._ok(err, "cudaMemcpy")
        return int(buf[0])

    def close(self) -> None:
        """Every rank: unmap the peers' buffers, then free its own once no
        peer maps them any more."""
        self.torch.cuda.synchronize()
        self.dist.barrier()
        for p in self.opened:
            self.rt.cudaIpcCloseMemHandle(p)
        self.opened = []
        self.dist.barrier()
        for p in self.local.values():
            self.rt.cudaFree(p)
        self.local = {}


class _DeviceFloats:
    """float32 device memory of `n` elements at `ptr`, for torch.as_tensor."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": "<f4", "data": (int(ptr), False),
                                         "version": 3}

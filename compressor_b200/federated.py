"""Federated round over several GPUs: host-side plan of the server step.

Clients are independent units (the codec keys all encoder and decoder state
by client id, reference momentum_compressor_openmp_simd_final.c:452-471), so
they are block-distributed over the ranks, one process per GPU.  Each rank
compresses its clients' updates, decodes them on its server-side decoder
instance with the weighted aggregate fused into the decode
(``falcom_set_aggregate``), and one sum all-reduce of the flat aggregate over
NCCL finishes the global update.

Everything here is plain host logic (which clients a rank owns, their
weights, the aggregate layout and the collective); it runs the same under the
``gloo`` backend on CPU tensors.
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


def layer_chunks(numels: Sequence[int], n_chunks: int) -> List[tuple]:
    """Splits items 0..len(numels)-1, in order, into at most n_chunks
    contiguous runs [i0, i1) of about equal element counts (a run ends once
    it reaches its share of the total; every run holds at least one item)."""
    n = len(numels)
    if n == 0:
        return []
    n_chunks = max(1, min(int(n_chunks), n))
    total = float(sum(int(x) for x in numels))
    out, i0, acc = [], 0, 0
    for i, x in enumerate(numels):
        acc += int(x)
        left_items, left_chunks = n - (i + 1), n_chunks - len(out) - 1
        if left_chunks > 0 and (acc >= total * (len(out) + 1) / n_chunks or left_items == left_chunks):
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

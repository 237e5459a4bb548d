"""CPU tests of the multi-GPU host logic (compressor_b200.federated): client
sharding, FedAvg weights, the flat aggregate layout, and the sum all-reduce
that finishes a federated round — run as world_size-2 gloo ranks."""
import os
import socket

import numpy as np
import pytest

from compressor_b200 import federated as F

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (16, 8), (5, 2), (3, 4), (0, 2), (7, 3)])
def test_shard_covers_every_client_once(n, world):
    owned = [c for r in range(world) for c in F.shard(n, world, r)]
    assert owned == list(range(n))
    sizes = [len(F.shard(n, world, r)) for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        F.shard(4, 2, 2)
    with pytest.raises(ValueError):
        F.uniform_weights(0)


def test_layout_offsets():
    lay = F.AggregateLayout.of(["a", "b", "c"], [(3, 2), (5,), (2, 2, 1, 1)], align=4)
    assert lay.offsets == [0, 8, 16] and lay.total == 20
    assert list(lay.c_offsets()) == [0, 8, 16]


def _decoded(client, rnd, total):
    """Stand-in for a decoded client update (deterministic per client)."""
    rng = np.random.default_rng(1000 * client + rnd)
    return (rng.standard_normal(total) * 1e-3).astype(np.float32)


def _worker(rank, world, port, n_clients, total, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = F.uniform_weights(n_clients)
        agg = torch.zeros(total, dtype=torch.float32)
        for c in F.shard(n_clients, world, rank):
            agg += w[c] * torch.from_numpy(_decoded(c, 0, total))
        F.allreduce_aggregate(agg, dist)
        np.save(f"{out_path}.{rank}.npy", agg.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n_clients", [6, 5])
def test_gloo_allreduce_equals_serial_fedavg(tmp_path, n_clients):
    import torch.multiprocessing as mp
    world, total = 2, 10_000
    out = str(tmp_path / "agg")
    mp.start_processes(_worker, args=(world, _free_port(), n_clients, total, out), nprocs=world,
                       join=True, start_method="spawn")
    serial = np.zeros(total, np.float64)
    for c in range(n_clients):
        serial += _decoded(c, 0, total).astype(np.float64) / n_clients
    got = [np.load(f"{out}.{r}.npy") for r in range(world)]
    assert np.array_equal(got[0], got[1])            # every rank holds the same global update
    assert np.max(np.abs(got[0] - serial)) <= 1e-9


def test_layer_chunks_cover_items_in_order():
    for numels, g in [([5, 1, 1, 1, 10, 2], 3), ([1] * 5, 8), ([100, 1, 1], 3), ([7], 4), ([3, 3, 3, 3], 2)]:
        ch = F.layer_chunks(numels, g)
        assert ch[0][0] == 0 and ch[-1][1] == len(numels)
        assert all(a[1] == b[0] for a, b in zip(ch, ch[1:]))
        assert all(i1 > i0 for i0, i1 in ch) and len(ch) <= g
    assert F.layer_chunks([3, 3, 3, 3], 2) == [(0, 2), (2, 4)]
    assert F.layer_chunks([], 3) == []
    # shares: a run ends once the cumulative share is reached
    assert F.layer_chunks([1] * 12, 3, fracs=[1, 2, 3]) == [(0, 2), (2, 6), (6, 12)]
    assert F.layer_chunks([5, 1, 1, 1], 2, fracs=[1, 1]) == [(0, 1), (1, 4)]
    assert F.layer_chunks([1, 1], 2, fracs=[1, 100, 100]) == [(0, 1), (1, 2)]
    with pytest.raises(ValueError):
        F.layer_chunks([1, 1], 2, fracs=[1, 0])


def _chunked_worker(rank, world, port, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shapes = [(64, 3, 3, 3), (64,), (128, 64, 1, 1), (10, 7), (5,), (256, 128, 3, 3)]
        lay = F.AggregateLayout.of([f"t{i}" for i in range(len(shapes))], shapes, align=4)
        agg = torch.from_numpy(_decoded(rank, 1, lay.total))
        whole = agg.clone()
        F.allreduce_aggregate(whole, dist)
        ar = F.ChunkedAllreduce(agg, lay, F.layer_chunks([int(np.prod(s)) for s in shapes], 3), dist)
        for c in range(len(ar.regions)):
            ar.chunk_done(c)
        ar.wait()
        ok = all(torch.equal(agg[o:o + int(np.prod(s))], whole[o:o + int(np.prod(s))])
                 for o, s in zip(lay.offsets, shapes))
        np.save(f"{out_path}.{rank}.npy", np.array([ok, len(ar.regions)]))
    finally:
        dist.destroy_process_group()


def test_gloo_chunked_allreduce_equals_whole(tmp_path):
    """The aggregate all-reduced one layer chunk at a time (asynchronous
    collectives, waited at the end) equals one all-reduce of the whole
    aggregate on every item, on every rank."""
    import torch.multiprocessing as mp
    world = 2
    out = str(tmp_path / "chunked")
    mp.start_processes(_chunked_worker, args=(world, _free_port(), out), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        ok, n = np.load(f"{out}.{r}.npy")
        assert ok and n == 3

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

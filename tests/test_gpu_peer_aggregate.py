"""GPU test of the two NVLink peer-memory sums of the server aggregate on
two GPUs (skipped with fewer), against NCCL's all-reduce of the same
per-rank aggregates: "fused", the reduce-scatter of the cross-GPU sum fused
into the decoder (falcom_set_aggregate_shards), then each rank's shard sum
and all-gather (falcom_shard_reduce); "oneshot", local aggregates, then
each rank's one-shot in-place all-reduce of its shard
(falcom_peer_allreduce) between NCCL barriers; "synced", the same with the
barriers on peer flag words inside the kernel
(falcom_peer_allreduce_sync).

Two ranks, one process per GPU (spawned, NCCL on 127.0.0.1).  Rank r
compresses two clients and decodes them on its server: the first into its
local aggregate (store mode), the second added to it (fused mode: landed in the
owners' slots).  A second server on each rank decodes the same payloads into
a plain local aggregate, which NCCL then all-reduces.  With two ranks both
sums add the same two float32 values, so the aggregates must be equal bit
for bit on both ranks, for three rounds (round 0 direct, then momentum)."""
import ctypes
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

NAMES = ["l1.conv.weight", "l1.bn.bias", "l2.conv.weight", "fc.weight", "fc.bias"]
SHAPES = [(64, 32, 3, 3), (64,), (128, 64, 1, 1), (10, 512), (10,)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, lib_path, out_dir, mode):
    import datetime
    import torch.distributed as dist
    from compressor_b200 import federated as F
    from compressor_b200.abi import Codec, PreparedBatch

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    lay = F.AggregateLayout.of(NAMES, SHAPES, align=64)
    offs_b = [4 * o for o in lay.offsets]
    c_offs = lay.c_offsets()
    peer = F.PeerAggregate(torch, dist, lay.total, rank, mode=mode)
    plain = torch.zeros(lay.total, dtype=torch.float32, device=dev)

    def mk(cid):
        c = Codec(lib_path, client=cid, param_count_threshold=16)
        c.lib.falcom_set_stream(c.h, ctypes.c_void_p(stream.cuda_stream))
        return c
    clients = [f"c{rank}_{k}" for k in range(2)]
    encs = {c: mk(c) for c in clients}
    srv, ref = mk("server"), mk("server")
    for c in (srv, ref):
        c.lib.falcom_set_aggregate_only(c.h, 1)
    w = 0.25
    pbs = {c: PreparedBatch(srv.lib, NAMES, SHAPES) for c in clients}
    rng = np.random.default_rng(100 + rank)
    ok = True
    for t in range(3):
        for k, cid in enumerate(clients):
            x = np.zeros(lay.total, np.float32)
            for o, s in zip(lay.offsets, SHAPES):
                n = int(np.prod(s))
                x[o:o + n] = rng.standard_normal(n).astype(np.float32) * 1e-3
            xd = torch.from_numpy(x).to(dev)
            torch.cuda.synchronize()
            pb = pbs[cid]
            pb.set_pointers(xd.data_ptr(), offs_b)
            assert pb.compress(encs[cid].h, cid.encode()) == 0
            for server, agg in ((srv, peer.agg), (ref, plain)):
                assert server.lib.falcom_set_aggregate(server.h, ctypes.c_void_p(agg.data_ptr()), c_offs,
                                                       len(NAMES), w) == 0
                assert server.lib.falcom_set_aggregate_store(server.h, 1 if k == 0 else 0) == 0
            if k == len(clients) - 1:
                peer.enable(srv.lib, srv.h)
            else:
                peer.disable(srv.lib, srv.h)
            assert pb.decompress(srv.h, cid.encode()) == 0
            assert pb.decompress(ref.h, cid.encode()) == 0
            pb.release()
        peer.finish(srv.lib, stream.cuda_stream)
        dist.all_reduce(plain)
        torch.cuda.synchronize()
        a, b = peer.agg.cpu().numpy(), plain.cpu().numpy()
        ok = ok and np.array_equal(a.view(np.uint32), b.view(np.uint32)) and peer.errors() == 0
    for c in list(encs.values()) + [srv, ref]:
        c.close()
    peer.close()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write("ok" if ok else "mismatch")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["fused", "oneshot", "synced"])
def test_peer_aggregate_equals_nccl_allreduce(product_lib, tmp_path, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), product_lib, str(tmp_path), mode), nprocs=2, join=True)
    for r in range(2):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok", r

"""Host logic of bench.py that needs no GPU: the choice of the cross-GPU sum
after the trial rounds, the e2e layer chunks and the e2e link bound."""
import numpy as np

import bench
from compressor_b200 import federated as F
from compressor_b200 import workloads as W


def test_choose_aggregate_fastest_passing():
    trial = {"peer": 0.71, "oneshot": 0.70, "synced": 0.67, "nccl": 0.74}
    assert bench.choose_aggregate(trial, {m: True for m in trial}) == "synced"
    # a mode whose FedAvg check failed is never chosen, however fast
    assert bench.choose_aggregate(trial, {"peer": True, "oneshot": True, "synced": False, "nccl": True}) == "oneshot"
    # a tie goes to the same mode on every rank (name order), whatever the dict order
    assert bench.choose_aggregate({"oneshot": 0.8, "nccl": 0.8}, {"oneshot": True, "nccl": True}) == "nccl"
    assert bench.choose_aggregate({"nccl": 0.8, "oneshot": 0.8}, {"oneshot": True, "nccl": True}) == "nccl"
    # nothing passed (or nothing ran): NCCL
    assert bench.choose_aggregate(trial, {}) == "nccl"
    assert bench.choose_aggregate({}, {}) == "nccl"


def test_e2e_chunks_cover_resnet50_in_order():
    lay = W.Layout.of("resnet50")
    numels = [int(np.prod(s)) for s in lay.shapes]
    ch = F.layer_chunks(numels, 3)
    assert ch[0][0] == 0 and ch[-1][1] == len(numels)
    assert all(a[1] == b[0] for a, b in zip(ch, ch[1:]))
    sizes = [sum(numels[a:b]) for a, b in ch]
    assert len(ch) == 3 and max(sizes) < 0.5 * sum(numels)


def test_e2e_link_bound():
    pcie = {"h2d_gbs": 50.0, "d2h_gbs": 50.0, "duplex_gbs": 80.0}
    # 1 GB each way: 20 ms alone per direction, 25 ms sharing the link
    assert abs(bench.e2e_link_bound(1e9, 1e9, pcie) - 25.0) < 1e-9
    # one direction only: its own rate binds
    assert abs(bench.e2e_link_bound(1e9, 0.0, pcie) - 20.0) < 1e-9
    assert abs(bench.e2e_link_bound(0.0, 2e9, pcie) - 40.0) < 1e-9

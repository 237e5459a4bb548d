#!/usr/bin/env python
"""Benchmark of the B200 FalCom codec.

Headline step (every N): one federated round with one client per GPU, the
ResNet-50 closed loop (266 tensors, 23,573,952 fp32, residual codec q8):
momentum_compressor_compress_batch on the client's encoder instance, then
momentum_compressor_decompress_batch on a separate server decoder instance
that writes the decoded update straight into the server's aggregate (weight
1/N, fused into the reconstruct kernel, aggregate-only: no separate decoded
copy), then, for N > 1, the NCCL sum all-reduce of the 94.3 MB aggregate.  At
N = 1 the weight is 1 and the aggregate is the decoded update itself, bit for
bit: the single-client closed loop.  Same step at every N (weak scaling).

  value    raw-update GB/s over all ranks (N x 94.3 MB / device time of the
           step, max over ranks), inputs resident in HBM
  e2e      the same step with host buffers: pinned host inputs, payloads
           returned to host memory and sent back up to the server, the
           aggregate read back to host memory, copies inside the timed step
  roofline dominant kernel: algorithmic bytes per launch / mean launch time
           (CUDA events on the library's stream), against the measured HBM
           copy bandwidth
  cpu_baseline  the reference's own grouped OpenMP codec (built from its
           sources, SZ3 stubbed) on the same workload on this host's cores

Nested lines: ``federated_64`` (64 ResNet-50 clients over the N GPUs, 64/N
per GPU, NCCL aggregate checked against a float64 FedAvg), ``gpt2_medium_16``
(16 GPT-2-medium clients, q8), and at N = 1 ``resnet18``, ``int4``,
``microbench_512x512x3x3`` (per-kernel GB/s beside the reference's own
microbenchmark), ``per_layer_api`` (the path FalComC.py calls),
``reference_gpu_v4`` (the reference's q8 GPU codec built for sm_100a),
``pcie`` and the CPU baseline at 8 threads and at all host threads.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "ResNet-50 closed-loop codec ms/round; raw-update GB/s/GPU vs HBM roofline"
PEAK_FALLBACK_GBS = 6650.0

# dram__bytes_read.sum + dram__bytes_write.sum per launch of each kernel, from
# one ncu capture of this bench (ResNet-50, q8, steady-state round); the
# capture summary and its command are committed under profiles/.  Re-captured
# whenever a kernel changes; None for workloads that were not captured.
NCU_TRAFFIC = {
    ("resnet50", "q8"): {
        "enc_pass3_predict": 342_665_216,
        "enc_pass4_quantize_pack": 201_046_528,
        "dec_prefix": 259_840,
        "dec_reconstruct": 439_436_032,
    },
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ----------------------------------------------------------------- helpers
def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return PEAK_FALLBACK_GBS, "fallback"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of the given GPUs, sampled by one
    process during a timed region (rank 0 samples every local GPU)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus, interval_ms: int = 20, enabled: bool = True):
        self.gpus = ",".join(str(g) for g in gpus)
        self.interval = interval_ms
        self.enabled = enabled
        self.proc = None
        self.lines = []

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpus, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.time()   # sampling is running once the first line is in
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.005)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            # a short timed region can end before the next sample: wait for
            # one more (taken as the region ends) before stopping
            n0, t0 = len(self.lines), time.time()
            while len(self.lines) <= n0 and time.time() - t0 < 1.0:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "gpus": self.gpus}


class L2Flush:
    """Empties the L2 between timed steps, outside the timed events: a 256 MiB
    write (no line of the previous step survives), then a 256 MiB read of a
    second buffer, which evicts the write's dirty lines too, so no write-back
    of the flush itself lands inside the next timed step."""

    def __init__(self, torch, device):
        n = 256 * 1024 * 1024 // 4
        self.w = torch.empty(n, dtype=torch.float32, device=device)
        self.r = torch.zeros(n, dtype=torch.float32, device=device)

    def __call__(self):
        self.w.zero_()
        self.r.sum()


class DevView:
    """Zero-copy torch view of float32 device memory the library owns (the
    CUDA array interface), for checks on decoded arrays."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": "<f4", "data": (int(ptr), False),
                                         "version": 3}


# ------------------------------------------------------------ distributed
class Dist:
    """One process per GPU under torchrun (NCCL); a single process otherwise."""

    def __init__(self):
        import torch
        self.torch = torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        # one stream for everything: torch's work (data, flushes, checks,
        # events) and the library's (falcom_set_stream), so every step is
        # ordered on it; the legacy default stream would leave the library
        # on its own non-blocking stream, unordered with torch's work
        self.stream = torch.cuda.Stream(device=self.dev)
        torch.cuda.set_stream(self.stream)
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
            self.dist = dist

    def barrier(self):
        """Host-side alignment of the ranks (device idle on both sides)."""
        self.torch.cuda.synchronize()
        if self.dist:
            self.dist.barrier()
            self.torch.cuda.synchronize()

    def max(self, x: float) -> float:
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device=self.dev)
        if self.dist:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum_(self, t):
        if self.dist:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)

    def close(self):
        if self.dist:
            self.dist.barrier()
            self.dist.destroy_process_group()


# ---------------------------------------------------------- synthetic data
class DeviceUpdates:
    """Seeded synthetic client updates generated on the GPU, one flat float32
    buffer per client in the model's packed layout (offsets aligned to 64
    elements).  ResNet / microbench: AR(1) Gaussian (rho 0.9, sigma
    1e-3/sqrt(fan_in), or 1e-4 for the microbench tensor); GPT-2-medium:
    Student-t nu = 3 scaled by 1e-4, rho 0.8 (t = z0 / sqrt((z1^2+z2^2+z3^2)/3));
    `common_std` > 0 adds a shared N(0, common_std^2) component drawn once per
    round with the same seed on every rank."""

    def __init__(self, torch, model: str, clients, dev, common_std: float = 0.0, seed0: int = 50_000):
        from compressor_b200 import workloads as W
        self.torch = torch
        self.lay = W.Layout.of(model)
        self.student = model == "gpt2-medium"
        self.rho = 0.8 if self.student else 0.9
        lay = self.lay
        self.sigma = torch.zeros(lay.total, device=dev)
        for o, sh in zip(lay.offsets, lay.shapes):
            n = int(np.prod(sh))
            s = 1e-4 if (self.student or model == "microbench") else 1e-3 / float(np.sqrt(W.fan_in(sh)))
            self.sigma[o:o + n] = s
        self.gens = []
        for c in clients:
            g = torch.Generator(device=dev)
            g.manual_seed(seed0 + int(c))
            self.gens.append(g)
        self.common_std = common_std
        self.gcom = torch.Generator(device=dev)
        self.gcom.manual_seed(seed0 - 1)
        self.state = [torch.zeros(lay.total, device=dev) for _ in clients]
        self.x = [s if common_std == 0.0 else torch.empty(lay.total, device=dev) for s in self.state]
        self.started = False
        self.dev = dev

    def _noise(self, g):
        t = self.torch
        n = self.lay.total
        if not self.student:
            return t.randn(n, device=self.dev, generator=g).mul_(self.sigma)
        z = t.randn(4, n, device=self.dev, generator=g)
        chi = z[1].square_().add_(z[2].square_()).add_(z[3].square_()).div_(3.0).sqrt_()
        return z[0].div_(chi).mul_(self.sigma)

    def next_round(self):
        common = None
        if self.common_std:
            common = self.torch.randn(self.lay.total, device=self.dev, generator=self.gcom).mul_(self.common_std)
        for j, g in enumerate(self.gens):
            noise = self._noise(g)
            if self.started:
                self.state[j].mul_(self.rho).add_(noise)
            else:
                self.state[j].copy_(noise)
            if common is not None:
                self.torch.add(self.state[j], common, out=self.x[j])
            del noise
        self.started = True

    def ptrs(self):
        return [x.data_ptr() for x in self.x]


# ------------------------------------------------------------ the round
def choose_aggregate(trial_ms: dict, passed: dict) -> str:
    """The --aggregate mode to use after the trial rounds: the fastest (max
    over ranks of the median step) among the modes whose FedAvg check passed;
    NCCL when none did.  A mode missing from trial_ms fell back to NCCL at
    set-up and is not a candidate."""
    ok = [m for m in trial_ms if passed.get(m)]
    return min(ok, key=lambda m: (trial_ms[m], m)) if ok else "nccl"


# --aggregate modes that sum over NVLink peer memory, and their PeerAggregate mode
PEER_MODES = {"peer": "fused", "oneshot": "oneshot", "synced": "synced"}
COLLECTIVES = {"peer": "decoder stores into owner shards over NVLink peer memory, shard sum + all-gather kernel",
               "oneshot": "one-shot in-place all-reduce kernel over NVLink peer memory (peer loads of the "
                          "rank's shard, sum, peer stores)",
               "synced": "one-shot in-place all-reduce kernel over NVLink peer memory with its barriers on "
                         "peer flag words inside the kernel (no NCCL call per round)",
               "nccl": "nccl all-reduce"}


class FedRound:
    """One federated round on this rank: every local client's update through
    its own encoder instance (compress_batch), then through this rank's server
    decoder (decompress_batch) with the weighted aggregate fused into the
    reconstruct kernel (first client stored, the others added,
    aggregate-only: no separate decoded copy), then the NCCL sum all-reduce of
    the aggregate over the ranks (N > 1)."""

    def __init__(self, torch, D: Dist, model: str, clients, n_total: int, codec: str, stream, so_path,
                 host_inputs: bool = False, peer: str = "nccl"):
        from compressor_b200 import workloads as W
        from compressor_b200.abi import Codec, PreparedBatch
        self.torch, self.D, self.model = torch, D, model
        self.lay = W.Layout.of(model)
        self.clients = list(clients)
        self.cids = [f"Client{c + 1}".encode() for c in self.clients]
        self.w = 1.0 / float(n_total)
        self.stream = stream
        self.host_inputs = host_inputs

        def mk(cid):
            c = Codec(so_path, client=cid)
            assert c.lib.falcom_set_residual_codec(c.h, codec.encode()) == 0
            c.lib.falcom_set_stream(c.h, ctypes.c_void_p(stream.cuda_stream))
            return c
        self.encs = [mk(cid.decode()) for cid in self.cids]
        self.srv = mk("server")
        # one prepared batch per client, its input pointers set once (the
        # inputs stay in place from round to round)
        self.pbs = [PreparedBatch(self.srv.lib, self.lay.names, self.lay.shapes) for _ in self.cids]
        self.bound = [None] * len(self.cids)
        self.offs_b = [4 * o for o in self.lay.offsets]
        self.c_offs = (ctypes.c_size_t * len(self.lay.offsets))(*self.lay.offsets)
        self.peer = None
        self.collective = "none" if D.world == 1 else "nccl all-reduce"
        if peer in PEER_MODES and D.world > 1:
            from compressor_b200 import federated as F
            try:   # every rank succeeds or every rank raises (PeerAggregate agrees first)
                self.peer = F.PeerAggregate(torch, D.dist, self.lay.total, D.local, mode=PEER_MODES[peer])
                self.collective = COLLECTIVES[peer]
            except RuntimeError as e:
                log(f"peer aggregate unavailable, NCCL all-reduce instead: {e}")
        if self.peer is not None:
            self.agg = self.peer.agg
        else:
            self.agg = torch.zeros(self.lay.total, dtype=torch.float32, device=D.dev)
        self.upd = self.lay.numel * 4
        self.launches = 0
        self.payload = 0
        self.srv_state = None
        self.shard_on = False

    def close(self):
        for c in self.encs + [self.srv]:
            c.close()
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def codec_part(self, ptrs, outputs: bool = False, check64=None, count_payload: bool = False):
        """Compress + decode of every local client (queued on the stream,
        each call synchronous with the host).  With `outputs` the server also
        returns decoded device arrays, and `check64` (float64, aggregate
        layout) accumulates weight * decoded for the FedAvg check;
        `count_payload` adds up the payload bytes (host work kept out of the
        timed steps)."""
        lib, srv = self.srv.lib, self.srv
        if count_payload:
            self.payload = 0
        for j, cid in enumerate(self.cids):
            pb = self.pbs[j]
            if self.bound[j] != ptrs[j]:
                pb.set_pointers(ptrs[j], self.offs_b)
                self.bound[j] = ptrs[j]
            r1 = pb.compress(self.encs[j].h, cid)
            # the server's aggregate settings, changed only when they differ
            # (uniform weights: set once; the store flag for the first client)
            want = (self.agg.data_ptr(), self.w, 1 if j == 0 else 0, 0 if outputs else 1)
            if self.srv_state is None or self.srv_state[:2] != want[:2]:
                assert lib.falcom_set_aggregate(srv.h, ctypes.c_void_p(want[0]), self.c_offs,
                                                len(self.lay.offsets), want[1]) == 0
                self.srv_state = (want[0], want[1], None, None)
            if self.srv_state[2] != want[2]:
                lib.falcom_set_aggregate_store(srv.h, want[2])
            if self.srv_state[3] != want[3]:
                lib.falcom_set_aggregate_only(srv.h, want[3])
            self.srv_state = want
            if self.peer is not None:
                # the rank's last client lands its partial sum in the owners' slots
                last = j == len(self.cids) - 1
                if last and not self.shard_on:
                    self.peer.enable(lib, srv.h)
                elif not last and self.shard_on:
                    self.peer.disable(lib, srv.h)
                self.shard_on = last
            r2 = pb.decompress(srv.h, cid)
            if r1 != 0 or r2 != 0:
                raise RuntimeError(f"codec failed on rank {self.D.rank} client {cid}: {r1} {r2} "
                                   f"{self.encs[j].lib.falcom_last_error(self.encs[j].h)} "
                                   f"{lib.falcom_last_error(srv.h)}")
            if count_payload:
                self.payload += pb.payload_bytes()
            self.launches += (self.encs[j].lib.falcom_last_launches(self.encs[j].h) +
                              lib.falcom_last_launches(srv.h))
            if check64 is not None:
                for i, o in enumerate(self.lay.offsets):
                    a = pb.outs[i].contents
                    v = self.torch.as_tensor(DevView(a.data, a.total_size), device=self.D.dev)
                    check64[o:o + a.total_size].add_(v.double(), alpha=self.w)
                # the views are read on the stream before release hands the
                # arrays back to the library (ordered anyway: one stream)
                self.torch.cuda.current_stream().synchronize()
            pb.release()

    def allreduce(self):
        if self.peer is not None:
            self.peer.finish(self.srv.lib, self.stream.cuda_stream)
        else:
            self.D.sum_(self.agg)


class E2ERound:
    """The headline step from host buffers, through the same public calls,
    pipelined over C layer chunks (contiguous layers of about equal size;
    the codec's state is per layer, so chunking changes no result).

    `xfer` = "sm" (the default) or "ce": the step first queues the uploads
    of every chunk's pinned host inputs on an upload stream, one event per
    chunk, so the host-to-device link streams the whole update while the
    codec works; chunk c's compress_batch (on the device copy, payloads
    returned in host memory) waits only for chunk c's upload.  "sm" moves the
    inputs up and the aggregate down with falcom_copy_sm (kernels, no copy
    engine), so the small copies the codec calls queue on the copy engines
    never wait behind them; "ce" with copy-engine copies.  "lib":
    compress_batch reads the pinned host inputs itself and uploads them
    inside the call.  Then chunk c's decompress_batch on the server (the
    payloads go up again and decode into the aggregate), for N > 1 the sum
    all-reduce of the chunk's aggregate region, and the download of that
    region on a side stream: the link carries data both ways at once."""

    XFER = ("sm", "ce", "lib")

    def __init__(self, torch, D: Dist, model: str, codec: str, stream, so_path, n_chunks: int,
                 xfer: str = "sm", fracs=None, down_blocks: int = 4, up_blocks: int = 0):
        from compressor_b200 import federated as F
        from compressor_b200 import workloads as W
        from compressor_b200.abi import Codec, PreparedBatch
        self.torch, self.D, self.stream = torch, D, stream
        self.lay = lay = W.Layout.of(model)
        self.cid = f"Client{D.rank + 1}".encode()
        self.w = 1.0 / D.world

        def mk(cid):
            c = Codec(so_path, client=cid)
            assert c.lib.falcom_set_residual_codec(c.h, codec.encode()) == 0
            c.lib.falcom_set_stream(c.h, ctypes.c_void_p(stream.cuda_stream))
            return c
        self.enc, self.srv = mk(self.cid.decode()), mk("server")
        self.chunks = F.layer_chunks([int(np.prod(sh)) for sh in lay.shapes], n_chunks, fracs)
        # falcom_copy_sm CTAs of the uploads (0: the library's default) and
        # of the aggregate downloads: few download CTAs leave the
        # device-to-host link to the payload copies of the next chunk's
        # compress_batch, which are on the critical path
        self.down_blocks, self.up_blocks = down_blocks, up_blocks
        self.pbs, self.offs_b, self.c_offs, self.regions = [], [], [], []
        for i0, i1 in self.chunks:
            self.pbs.append(PreparedBatch(self.srv.lib, lay.names[i0:i1], lay.shapes[i0:i1]))
            self.offs_b.append([4 * o for o in lay.offsets[i0:i1]])
            self.c_offs.append((ctypes.c_size_t * (i1 - i0))(*lay.offsets[i0:i1]))
            last = i1 - 1
            self.regions.append((lay.offsets[i0], lay.offsets[last] + int(np.prod(lay.shapes[last]))))
        self.agg = torch.zeros(lay.total, dtype=torch.float32, device=D.dev)
        self.agg_host = torch.empty(lay.total, dtype=torch.float32, pin_memory=True)
        self.side = torch.cuda.Stream(device=D.dev)
        if xfer not in self.XFER:
            raise ValueError(f"unknown e2e transfer mode {xfer!r}")
        self.xfer = xfer
        self.prefetch = xfer != "lib"
        if self.prefetch:
            self.up = torch.cuda.Stream(device=D.dev)
            self.dev_in = torch.empty(lay.total, dtype=torch.float32, device=D.dev)
        self.upd = lay.numel * 4
        self.payload = 0
        self.sm_copies = 0
        if xfer == "sm":   # pinned memory that is not mapped into the device address space: copy engines
            probe = torch.empty(4, dtype=torch.float32, pin_memory=True)
            rc = self.srv.lib.falcom_copy_sm(ctypes.c_void_p(self.agg.data_ptr()), ctypes.c_void_p(probe.data_ptr()),
                                             16, 0, ctypes.c_void_p(stream.cuda_stream))
            torch.cuda.current_stream().synchronize()
            if rc != 0:
                log(f"falcom_copy_sm refused pinned memory ({rc}); e2e transfers by copy engines")
                self.xfer = "ce"

    def step(self, host, count_payload: bool = False):
        """One round from the pinned float32 host tensor `host` (the flat
        update in the layout's offsets)."""
        torch, lib, srv = self.torch, self.srv.lib, self.srv
        if count_payload:
            self.payload = 0
        if self.prefetch:
            # the previous round's compress calls have returned, so the
            # device copy is free once the stream's earlier work is done
            self.up.wait_stream(self.stream)
            ready = []
            with torch.cuda.stream(self.up):
                for lo, hi in self.regions:
                    self._move(self.dev_in[lo:hi], host[lo:hi], self.up, self.up_blocks)
                    ev = torch.cuda.Event()
                    ev.record(self.up)
                    ready.append(ev)
            src = self.dev_in.data_ptr()
        else:
            src = host.data_ptr()
        for c, pb in enumerate(self.pbs):
            if self.prefetch:
                self.stream.wait_event(ready[c])
            pb.set_pointers(src, self.offs_b[c])
            r1 = pb.compress(self.enc.h, self.cid)
            assert lib.falcom_set_aggregate(srv.h, ctypes.c_void_p(self.agg.data_ptr()), self.c_offs[c],
                                            len(self.offs_b[c]), self.w) == 0
            lib.falcom_set_aggregate_store(srv.h, 1)
            lib.falcom_set_aggregate_only(srv.h, 1)
            r2 = pb.decompress(srv.h, self.cid)
            if r1 != 0 or r2 != 0:
                raise RuntimeError(f"codec failed (e2e chunk {c}): {r1} {r2}")
            if count_payload:
                self.payload += pb.payload_bytes()
            pb.release()
            lo, hi = self.regions[c]
            self.D.sum_(self.agg[lo:hi])
            ev = torch.cuda.Event()
            ev.record(self.stream)
            self.side.wait_event(ev)
            with torch.cuda.stream(self.side):
                self._move(self.agg_host[lo:hi], self.agg[lo:hi], self.side, self.down_blocks)
        self.stream.wait_stream(self.side)
        if self.prefetch:
            self.stream.wait_stream(self.up)

    def _move(self, dst, src, stream, blocks: int = 0):
        """dst <- src (float32, one of them pinned host memory) on `stream`."""
        if self.xfer == "sm":
            rc = self.srv.lib.falcom_copy_sm(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src.data_ptr()),
                                             4 * src.numel(), blocks, ctypes.c_void_p(stream.cuda_stream))
            if rc != 0:
                raise RuntimeError(f"falcom_copy_sm failed ({rc})")
            self.sm_copies += 1
        else:
            dst.copy_(src, non_blocking=True)

    def close(self):
        self.enc.close()
        self.srv.close()


def timed_rounds(torch, D: Dist, fr: FedRound, data: DeviceUpdates, K: int, W: int, flush, clk=None,
                 split: bool = False):
    """W untimed rounds, then K rounds each bracketed by CUDA events on the
    library's stream (L2 flush and rank alignment outside them).  Returns
    per-step ms, codec-part ms and all-reduce ms (rank-local)."""
    stream = fr.stream
    for w in range(W):
        data.next_round()
        fr.codec_part(data.ptrs(), count_payload=(w == W - 1))
        fr.allreduce()
    torch.cuda.synchronize()
    step, codec, ar, wait = [], [], [], []
    fr.launches = 0
    tiny = torch.zeros(1, device=D.dev)
    for _ in range(K):
        data.next_round()
        # ranks aligned on the host first; the flush that follows gives the
        # host time to plan the step's first call while the GPU is still busy
        D.barrier()
        flush()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        e[0].record(stream)
        fr.codec_part(data.ptrs())
        e[1].record(stream)
        if split:
            D.sum_(tiny)             # completes once every rank has arrived
        e[2].record(stream)
        fr.allreduce()
        e[3].record(stream)
        e[3].synchronize()
        step.append(e[0].elapsed_time(e[3]))
        codec.append(e[0].elapsed_time(e[1]))
        wait.append(e[1].elapsed_time(e[2]))
        ar.append(e[2].elapsed_time(e[3]))
    torch.cuda.synchronize()
    return step, codec, wait, ar


def e2e_link_bound(h2d_bytes: float, d2h_bytes: float, pcie: dict) -> float:
    """Lower bound in ms of an e2e step's host transfers from the pinned copy
    rates measured in the same run: the slower of the upload alone, the
    download alone, and both directions sharing the link at their measured
    combined rate."""
    up = h2d_bytes / (pcie["h2d_gbs"] * 1e9)
    down = d2h_bytes / (pcie["d2h_gbs"] * 1e9)
    both = (h2d_bytes + d2h_bytes) / (pcie["duplex_gbs"] * 1e9)
    return 1e3 * max(up, down, both)


def first_rounds(torch, D: Dist, model, world, codec, stream, so, aggregate, flush, hot_steps):
    """Rounds 0, 1 and 2 of fresh encoder / decoder instances, each timed
    like a hot step (L2 flushed before it, CUDA events, max over ranks),
    beside the median of the hot steps.  Round 0 has no history: every
    tensor takes the direct path and the state is allocated; round 1 is the
    first momentum round (the previous gradient's statistics not yet
    known); from round 2 on the rounds are hot."""
    fr0 = FedRound(torch, D, model, [D.rank], world, codec, stream, so, peer=aggregate)
    d0 = DeviceUpdates(torch, model, [D.rank], D.dev, seed0=1500)
    s0, _, _, _ = timed_rounds(torch, D, fr0, d0, 3, 0, flush)
    fr0.close()
    del d0
    return {"round0_ms": round(D.max(s0[0]), 4), "round1_ms": round(D.max(s0[1]), 4),
            "round2_ms": round(D.max(s0[2]), 4), "hot_median_ms": round(D.max(statistics.median(hot_steps)), 4),
            "how": "fresh instances, rounds 0-2 timed like the hot steps (L2 flushed before each, CUDA events, "
                   "max over ranks); round 0: no history, every tensor direct, state allocated; round 1: first "
                   "momentum round; hot median: the timed steps of the headline"}


def fedavg_check(torch, D: Dist, fr: FedRound, data: DeviceUpdates):
    """One more round in which the server also returns the decoded arrays:
    rank 0 compares the NCCL-reduced float32 aggregate with the float64 sum
    over all clients of weight * decoded (all-reduced in float64)."""
    acc = torch.zeros(fr.lay.total, dtype=torch.float64, device=D.dev)
    data.next_round()
    fr.codec_part(data.ptrs(), outputs=True, check64=acc)
    fr.allreduce()
    D.sum_(acc)
    torch.cuda.synchronize()
    a = fr.agg.double()
    num = float(torch.linalg.vector_norm(a - acc).item())
    den = float(torch.linalg.vector_norm(acc).item())
    exact = bool(torch.equal(fr.agg, acc.float())) if D.world == 1 and len(fr.clients) == 1 else None
    rel = num / den if den > 0 else num
    # synced peer mode: a barrier wait that ran out inside the kernel, on any rank
    sync_err = D.max(float(fr.peer.errors())) if fr.peer is not None else 0.0
    out = {"rel_l2": rel, "pass": rel <= 1e-6 and sync_err == 0.0, "bar": 1e-6, "bit_exact_single_client": exact,
           "against": "float64 sum over all clients of weight x decoded update (FedAvg), all-reduced in float64"}
    if fr.peer is not None and fr.peer.mode == "synced":
        out["barrier_timeouts"] = int(sync_err)
    return out


# ------------------------------------------------------------ reference CPU
def ref_library():
    from oracle import binding as ob
    if not ob.have_ref():
        return None
    return ob.REF_SO


def cpu_reference_loop(model: str, steps: int, warmup: int, threads: int, budget_s: float = None):
    """Closed loop of the reference grouped OpenMP codec on the host cores:
    compress_batch on an encoder instance, decompress_batch on a decoder
    instance, one round per step.  Returns per-step seconds."""
    os.environ.setdefault("OMP_PROC_BIND", "close")
    os.environ.setdefault("OMP_PLACES", "cores")
    os.environ.setdefault("FALCOM_LOG_LEVEL", "ERROR")
    from compressor_b200 import workloads as W
    from compressor_b200.abi import Codec, HostArray, NDArrayC
    so = ref_library()
    gomp = ctypes.CDLL("libgomp.so.1")
    gomp.omp_set_num_threads(int(threads))
    lay = W.Layout.of(model)
    n_distinct = 4
    data = W.rounds(model, n_distinct, seed=1234)
    enc = Codec(so, client="Client1")
    dec = Codec(so, client="Client1")
    names = lay.names
    times = []
    # silence the reference's per-call stdout/stderr lines
    devnull = os.open(os.devnull, os.O_WRONLY)
    saved = (os.dup(1), os.dup(2))
    os.dup2(devnull, 1)
    os.dup2(devnull, 2)
    try:
        t_start = time.perf_counter()
        for t in range(1 + warmup + steps):
            flat = data[t % n_distinct]
            hs = [HostArray(v) for v in lay.views(flat)]
            t0 = time.perf_counter()
            ret, items = enc.compress_batch_raw(names, hs)
            n = len(names)
            outs = (ctypes.POINTER(NDArrayC) * n)()
            r2 = dec.lib.momentum_compressor_decompress_batch(dec.h, items, n, b"Client1", outs)
            t1 = time.perf_counter()
            for i in range(n):
                if outs[i]:
                    dec.lib.ndarray_destroy(outs[i])
            enc.free_items(items)
            if ret != 0 or r2 != 0:
                raise RuntimeError(f"reference codec failed ({ret}, {r2})")
            if t >= 1 + warmup:
                times.append(t1 - t0)
            if budget_s and time.perf_counter() - t_start > budget_s and len(times) >= 1:
                break
        enc.close()
        dec.close()
    finally:
        sys.stdout.flush()
        os.dup2(saved[0], 1)
        os.dup2(saved[1], 2)
        os.close(devnull)
        os.close(saved[0])
        os.close(saved[1])
    return times


def update_bytes(model: str) -> int:
    from compressor_b200 import workloads as W
    return W.Layout.of(model).numel * 4


def cpu_baseline_entry(model: str, threads: int, budget_s: float):
    ct = cpu_reference_loop(model, 20, 1, threads, budget_s=budget_s)
    cms = 1e3 * statistics.median(ct)
    return {"value": round(update_bytes(model) / (cms * 1e-3) / 1e9, 5), "unit": "GB/s", "cores": threads,
            "kind": "reference", "ms_per_round": round(cms, 2), "cpu_model": cpu_model(),
            "host_threads_available": os.cpu_count(),
            "sample": f"{len(ct)} full {model} closed-loop rounds (compress_batch + decompress_batch) of the "
                      f"reference grouped OpenMP build, SZ3 stubbed (sz3_memcpy), OMP_PROC_BIND=close "
                      f"OMP_PLACES=cores, {threads} threads, median, after 1 warm-up round"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    so = ref_library()
    cfg = {"workload": f"{args.model} single-client closed loop (compress_batch + decompress_batch, "
                       f"separate encoder/decoder instances), reference grouped OpenMP codec, SZ3 stubbed "
                       f"(sz3_memcpy)", "tensors": 266 if args.model == "resnet50" else None,
           "elements": update_bytes(args.model) // 4}
    if so is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference build oracle/_ref missing"}))
        return 0
    threads = os.cpu_count() or 1
    times = cpu_reference_loop(args.model, args.steps, args.warmup, threads)
    ms = 1e3 * statistics.mean(times)
    gbs = update_bytes(args.model) / (ms * 1e-3) / 1e9
    out = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 5), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded AR(1) Gaussian updates, ResNet-50 state-dict shapes)", "config": cfg,
        "cpu_baseline": {"value": round(gbs, 5), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "cpu_model": cpu_model(),
                         "sample": f"{len(times)} full closed-loop rounds after {args.warmup} warm-up rounds"},
        "e2e": {"value": round(gbs, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))
    return 0


# ------------------------------------------------------------- sub-benches
def kernel_roofline(torch, D, fr: FedRound, data: DeviceUpdates, K: int, flush, codec: str):
    """Per-kernel CUDA-event times of the codec kernels over K more rounds
    (events bracket every launch inside the library), and the dominant
    kernel's algorithmic bytes per launch / mean launch time."""
    from compressor_b200 import workloads as Wl
    from compressor_b200.abi import kernel_times
    insts = fr.encs + [fr.srv]
    for c in insts:
        c.lib.falcom_set_kernel_timing(c.h, 1)
    for _ in range(K):
        data.next_round()
        flush()
        fr.codec_part(data.ptrs())
        fr.allreduce()
    torch.cuda.synchronize()
    tot = {}
    for c in insts:
        for k, v in kernel_times(c.lib, c.h).items():
            a = tot.get(k, (0.0, 0))
            tot[k] = (a[0] + v[0], a[1] + v[1])
        c.lib.falcom_set_kernel_timing(c.h, 0)
    ab = Wl.algorithmic_bytes(fr.model, codec)
    q = {"q8": 1.0, "int4": 0.5, "raw": 4.0}[codec]
    me, de = ab["momentum_elements"], ab["direct_elements"]
    nc = len(fr.clients)
    # algorithmic bytes per launch of each kernel (all kernels predicted,
    # steady state: the previous gradient's |x| statistics come from the
    # round that wrote it, so passes 1 and 2 do not read it); the decoder
    # writes memory, history and the aggregate (store mode: the old value is
    # not read; first client of a round)
    alg = {
        "enc_pass1_stats_sign": me * 8 + de * 8,           # read cur; write history copy
        "enc_pass2_variance": me * 4,                       # read cur
        "enc_pass3_predict": me * 16,                       # read cur, prev, mem; write mem
        "enc_pass4_quantize_pack": me * (8 + q) + de * (4 + q),   # read cur, mem; write codes
        "dec_reconstruct": me * (20 + q) + de * (8 + q),    # read q, prev, mem; write mem, history, aggregate
        "dec_prefix": ab["kernels"] / 8,
        "frames_expand": ab["kernels"] / 8 * 2 * 2,
    }
    shares = {k: v[0] for k, v in tot.items() if v[1] > 0}
    dom = max((k for k in shares if k in alg), key=shares.get)
    avg_ms = tot[dom][0] / tot[dom][1]
    achieved = alg[dom] / (avg_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    return {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
            "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": NCU_TRAFFIC.get((fr.model, codec), {}).get(dom),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one steady-state launch",
            "algorithmic_bytes_per_launch": int(alg[dom]), "avg_launch_ms": round(avg_ms, 5),
            "kernel_share": {k: round(v / sum(shares.values()), 4) for k, v in shares.items()},
            "kernel_ms_per_round": {k: round(v[0] / K, 5) for k, v in tot.items() if v[1] > 0},
            "launches_per_round": {k: round(v[1] / K, 2) for k, v in tot.items() if v[1] > 0},
            "kernel_gbs": {k: round(alg[k] * nc / (tot[k][0] / K * 1e-3) / 1e9, 1)
                           for k in alg if k in tot and tot[k][1] > 0},
            "closed_loop_algorithmic_bytes": int(ab["bytes_per_round"])}


def closed_loop_line(torch, D, model, codec, K, W, flush, so, stream):
    """Single-client closed loop (the headline step at N = 1) of another model
    or codec: ms per round and raw-update GB/s."""
    from compressor_b200 import workloads as Wl
    fr = FedRound(torch, D, model, [0], 1, codec, stream, so)
    data = DeviceUpdates(torch, model, [0], D.dev, seed0=7000)
    step, codec_ms, _, _ = timed_rounds(torch, D, fr, data, K, W, flush)
    ms = statistics.mean(step)
    ab = Wl.algorithmic_bytes(model, codec)
    peak, _ = measured_peak()
    out = {"ms_per_step": round(ms, 4), "value": round(fr.upd / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
           "steps": K, "warmup": W, "codec": codec, "elements": fr.lay.numel,
           "closed_loop_frac": round(ab["bytes_per_round"] / (ms * 1e-3) / 1e9 / peak, 4),
           "payload_bytes_per_round": fr.payload}
    fr.close()
    return out


def federated_line(torch, D, model, n_clients, codec, K, W, flush, so, stream, common_std, peer="nccl"):
    """n_clients clients block-distributed over the ranks; per step: every
    local client's compress + decode into the aggregate, then the NCCL
    all-reduce; value = all clients' update bytes / max-over-ranks step time.
    Ends with the FedAvg check of the reduced aggregate."""
    from compressor_b200 import federated as F
    mine = list(F.shard(n_clients, D.world, D.rank))
    fr = FedRound(torch, D, model, mine, n_clients, codec, stream, so, peer=peer)
    data = DeviceUpdates(torch, model, mine, D.dev, common_std=common_std)
    step, codec_ms, wait, ar = timed_rounds(torch, D, fr, data, K, W, flush, split=D.world > 1)
    total = D.max(sum(step))
    ms = total / K
    check = fedavg_check(torch, D, fr, data)
    out = {"ms_per_step": round(ms, 4), "value": round(n_clients * fr.upd / (ms * 1e-3) / 1e9, 3),
           "unit": "GB/s", "scaling": "strong", "clients": n_clients, "clients_per_gpu": len(mine),
           "steps": K, "warmup": W, "codec": codec, "elements_per_client": fr.lay.numel,
           "codec_ms_per_client_rank0": round(statistics.mean(codec_ms) / max(1, len(mine)), 4),
           "peer_wait_ms_rank0": round(statistics.mean(wait), 4) if D.world > 1 else 0.0,
           "allreduce_ms_rank0": round(statistics.mean(ar), 4) if D.world > 1 else 0.0,
           "allreduce_bytes": 4 * fr.lay.total if D.world > 1 else 0,
           "aggregate_collective": fr.collective,
           "aggregate_check": check, "gpu_launches_per_step_rank0": fr.launches // max(1, K)}
    fr.close()
    del data
    torch.cuda.empty_cache()
    return out


def microbench_line(torch, D, K, flush, so, stream, codec="q8"):
    """Config 3: one 512x512x3x3 fp32 tensor, N(0, (1e-4)^2) AR(1) rho 0.9
    updates, closed loop over K rounds; per-kernel CUDA-event times and GB/s
    of algorithmic bytes, beside the reference's own six-kernel
    microbenchmark built for sm_100a (oracle/_ref/falcom_cuda_microbench)
    when present."""
    from compressor_b200.abi import kernel_times
    fr = FedRound(torch, D, "microbench", [0], 1, codec, stream, so)
    data = DeviceUpdates(torch, "microbench", [0], D.dev, seed0=3000)
    step, _, _, _ = timed_rounds(torch, D, fr, data, K, 3, flush)
    insts = fr.encs + [fr.srv]
    for c in insts:
        c.lib.falcom_set_kernel_timing(c.h, 1)
    for _ in range(K):
        data.next_round()
        flush()
        fr.codec_part(data.ptrs())
    torch.cuda.synchronize()
    tot = {}
    for c in insts:
        for k, v in kernel_times(c.lib, c.h).items():
            a = tot.get(k, (0.0, 0))
            tot[k] = (a[0] + v[0], a[1] + v[1])
    n = 512 * 512 * 9
    kern = 512 * 512
    # algorithmic bytes per launch (all kernels predicted; from the third round on the previous
    # gradient's statistics are known, so passes 1 and 2 read only cur) and the reference
    # microbench kernels each of ours covers
    alg = {
        "enc_pass1_stats_sign": (8 * n + kern / 8 * 2, "threshold_scan + bitmap_pack (+ stats sums, history copy)"),
        "enc_pass2_variance": (4 * n, "(stats second pass)"),
        "enc_pass3_predict": (16 * n, "momentum_update + residual_predmem_update"),
        "enc_pass4_quantize_pack": (9 * n + kern / 8 * 2, "dominant_sign_pack (+ q8 codes, bitmap frame)"),
        "dec_reconstruct": (21 * n, "decompress_reconstruct (+ q8 decode, memory update)"),
    }
    kernels = {}
    for k, (b, covers) in alg.items():
        if k in tot and tot[k][1] > 0:
            ms = tot[k][0] / tot[k][1]
            kernels[k] = {"us_per_launch": round(ms * 1e3, 2), "algorithmic_bytes": int(b),
                          "gbs": round(b / (ms * 1e-3) / 1e9, 1), "covers": covers}
    out = {"ms_per_round": round(statistics.mean(step), 4), "rounds": K, "elements": n, "conv_kernels": kern,
           "l2": "flushed before every round", "kernels": kernels}
    fr.close()
    mb = os.path.join(ROOT, "oracle", "_ref", "falcom_cuda_microbench")
    if os.path.exists(mb):
        try:
            r = subprocess.run([mb, "--numel", str(n), "--iters", "200"], capture_output=True, text=True,
                               timeout=300)
            rows = {}
            lines = r.stdout.strip().splitlines()
            hdr = lines[0].split(",")
            for line in lines[1:]:
                v = dict(zip(hdr, line.split(",")))
                g = float(v["gpu_only_ms"])
                rows[v["kernel"]] = {"gpu_only_us": round(g * 1e3, 2), "cpu_ms": float(v["cpu_ms"]),
                                     "h2d_gpu_d2h_ms": float(v["h2d_gpu_d2h_ms"])}
            out["reference_microbench_b200"] = {
                "rows": rows, "rc": r.returncode,
                "how": "the reference's falcom_cuda_microbench.cu built for sm_100a, --numel 2359296 --iters "
                       "200: back-to-back launches on one resident 9.4 MB input (L2-resident on B200)"}
        except Exception as e:   # a missing or failing baseline does not stop the bench
            out["reference_microbench_b200"] = {"error": str(e)[:200]}
    return out


def per_layer_line(torch, so, rounds: int = 4):
    """The path FalComC.py drives (FalComC.py:545,659): 266 separate
    momentum_compressor_compress_layer calls on host arrays, then 266
    decompress_layer calls on a second instance; host wall time per round."""
    from compressor_b200 import workloads as W
    from compressor_b200.abi import Codec, HostArray
    lay = W.Layout.of("resnet50")
    data = W.rounds("resnet50", rounds + 2, seed=4321)
    enc, dec = Codec(so, client="Client1"), Codec(so, client="Client1")
    names = [nm.encode() for nm in lay.names]
    ts = []
    for t, flat in enumerate(data):
        hs = [HostArray(v) for v in lay.views(flat)]
        t0 = time.perf_counter()
        for i, nm in enumerate(names):
            p = enc.lib.momentum_compressor_compress_layer(enc.h, nm, ctypes.byref(hs[i].c))
            if not p:
                raise RuntimeError("compress_layer failed")
            o = dec.lib.momentum_compressor_decompress_layer(dec.h, p, b"Client1", nm)
            if not o:
                raise RuntimeError("decompress_layer failed")
            dec.lib.ndarray_destroy(o)
            enc.lib.compressed_layer_data_free(p)
        if t >= 2:
            ts.append(time.perf_counter() - t0)
    enc.close()
    dec.close()
    ms = 1e3 * statistics.median(ts)
    return {"ms_per_round": round(ms, 3), "value": round(lay.numel * 4 / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "calls_per_round": 2 * len(names), "rounds": len(ts),
            "how": "host wall clock; host float32 inputs, host payloads, host decoded arrays (FalComC's "
                   "memory kinds); compress_layer and decompress_layer per tensor"}


def pcie_line(torch, dev):
    """Pinned host <-> device copy bandwidth (256 MiB, CUDA events, best of 5),
    one direction at a time and both at once on two streams."""
    n = 256 * 1024 * 1024
    h1 = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    h2 = torch.empty(n, dtype=torch.uint8, pin_memory=True)
    d1 = torch.empty(n, dtype=torch.uint8, device=dev)
    d2 = torch.empty(n, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()

    def one(fn):
        best = 1e9
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        return best

    h2d = one(lambda: d1.copy_(h1, non_blocking=True))
    d2h = one(lambda: h2.copy_(d2, non_blocking=True))

    def both():
        cur = torch.cuda.current_stream()
        for s in (s1, s2):
            s.wait_stream(cur)
        with torch.cuda.stream(s1):
            d1.copy_(h1, non_blocking=True)
        with torch.cuda.stream(s2):
            h2.copy_(d2, non_blocking=True)
        cur.wait_stream(s1)
        cur.wait_stream(s2)
    duplex = one(both)
    return {"h2d_gbs": round(n / (h2d * 1e-3) / 1e9, 2), "d2h_gbs": round(n / (d2h * 1e-3) / 1e9, 2),
            "duplex_gbs": round(2 * n / (duplex * 1e-3) / 1e9, 2), "bytes": n}


def reference_v4_line(torch, dev, rounds: int = 5):
    """The reference's fused q8 GPU codec (cuda_feasibility/falcom_cuda_v4,
    encode_q8_batch / decode_q8_batch) built from its own sources for sm_100a
    (oracle/build_ref_gpu.py), on the same ResNet-50 rounds: encode of the
    266 device tensors against the previous round (delta q8, one host sync
    per layer, payload blob copied to pinned host memory), then decode from
    that blob.  Host wall clock per round, the way the reference times it."""
    import importlib.machinery
    import importlib.util
    so = os.path.join(ROOT, "oracle", "_ref", "v4", "_falcom_cuda_v4.so")
    if not os.path.exists(so):
        return {"unavailable": "oracle/_ref/v4 not built"}
    spec = importlib.util.spec_from_file_location("_falcom_cuda_v4", so,
                                                  loader=importlib.machinery.ExtensionFileLoader("_falcom_cuda_v4", so))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    data = DeviceUpdates(torch, "resnet50", [0], dev, seed0=8000)
    lay = data.lay
    shapes = [list(s) for s in lay.shapes]
    flags = torch.ones(len(shapes), dtype=torch.uint8)
    prev = None
    ts = []
    for t in range(rounds + 2):
        data.next_round()
        cur = [data.x[0][o:o + int(np.prod(s))].view(*s).clone() for o, s in zip(lay.offsets, lay.shapes)]
        if prev is not None:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            blob, offs, lens, scales, cands, _ = m.encode_q8_batch(cur, prev, flags)
            dec, _ = m.decode_q8_batch(blob, offs, lens, scales, shapes, prev, flags, dev.index or 0)
            torch.cuda.synchronize()
            if t >= 2:
                ts.append(time.perf_counter() - t0)
        prev = cur
    ms = 1e3 * statistics.median(ts)
    return {"ms_per_round": round(ms, 3), "value": round(lay.numel * 4 / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "rounds": len(ts),
            "how": "reference v4 encode_q8_batch + decode_q8_batch (delta q8 in its own envelope, not the C wire "
                   "format), device tensors in, pinned host blob between them, host wall clock"}


# ------------------------------------------------------------------- ours
def run_ours(args):
    import torch
    D = Dist()
    from compressor_b200 import build as B
    if not os.path.exists(B.OUT):
        B.build()
    os.environ.setdefault("FALCOM_LOG_LEVEL", "ERROR")
    so = B.OUT
    stream = D.stream
    assert stream.cuda_stream != 0
    flush = L2Flush(torch, D.dev)
    K, Wm = args.steps, args.warmup
    model, codec = args.model, args.codec
    world = D.world

    # ------------------------------------------------ headline (device value)
    # N > 1, --aggregate auto: both ways of summing the aggregate over the
    # GPUs run a few untimed rounds, and the faster (max over ranks) is used
    # for the timed rounds and the nested lines
    choice = None
    if world > 1 and args.aggregate == "auto":
        trial = {}
        checks = {}
        for mode in ("peer", "oneshot", "synced", "nccl"):
            ft = FedRound(torch, D, model, [D.rank], world, codec, stream, so, peer=mode)
            dt = DeviceUpdates(torch, model, [D.rank], D.dev, seed0=900)
            st_, _, _, _ = timed_rounds(torch, D, ft, dt, 8, 4, flush)
            # a mode whose sum fails the FedAvg check is not chosen
            ok = D.max(0.0 if fedavg_check(torch, D, ft, dt)["pass"] else 1.0) == 0.0
            if ft.collective == COLLECTIVES[mode]:     # not fallen back to NCCL
                trial[mode] = D.max(statistics.median(st_))
                checks[mode] = ok
            ft.close()
            del dt
        best = choose_aggregate(trial, checks)
        choice = {"chosen": best, "trial_ms_per_step": {m: round(v, 4) for m, v in trial.items()},
                  "trial_fedavg_pass": checks,
                  "how": "8 untimed rounds each after 4 warm-up rounds, median, max over ranks; then one "
                         "FedAvg-checked round"}
        args.aggregate = best
    fr = FedRound(torch, D, model, [D.rank], world, codec, stream, so, peer=args.aggregate)
    data = DeviceUpdates(torch, model, [D.rank], D.dev, seed0=1000)
    local_gpus = list(range(int(os.environ.get("LOCAL_WORLD_SIZE", world))))
    with ClockSampler(local_gpus, interval_ms=20 if world == 1 else 50, enabled=D.local == 0) as clk:
        step, codec_ms, _, ar = timed_rounds(torch, D, fr, data, K, Wm, flush)
    total_ms = D.max(sum(step))
    ms_per_step = total_ms / K
    value = world * fr.upd / (ms_per_step * 1e-3) / 1e9
    launches_timed = fr.launches
    payload = fr.payload
    if args.mode == "value":
        fr.close()
        if D.rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
                              "steps": K, "warmup": Wm, "ms_per_step": round(ms_per_step, 4),
                              "mode": "value-only (profiler run)"}))
        D.close()
        return 0
    codec_max = D.max(statistics.mean(codec_ms))
    # peer wait vs transfer of the all-reduce, in separate diagnostic rounds
    split = None
    if world > 1:
        s2, c2, w2, a2 = timed_rounds(torch, D, fr, data, min(K, 10), 0, flush, split=True)
        split = {"steps": len(s2), "peer_wait_ms_rank0": round(statistics.mean(w2), 4),
                 "transfer_ms_rank0": round(statistics.mean(a2), 4),
                 "transfer_ms_max": round(D.max(statistics.mean(a2)), 4),
                 "how": "a 1-element all-reduce after the decode ends when every rank has arrived (peer wait); "
                        "the aggregate all-reduce follows (transfer); rounds outside the timed ones"}
    roofline = kernel_roofline(torch, D, fr, data, K, flush, codec)
    peak = roofline["peak"]
    roofline["closed_loop_frac"] = round(roofline["closed_loop_algorithmic_bytes"] /
                                         (codec_max * 1e-3) / 1e9 / peak, 4)
    check = fedavg_check(torch, D, fr, data)
    collective = fr.collective
    fr.close()
    first = first_rounds(torch, D, model, world, codec, stream, so, args.aggregate, flush, step)

    # ------------------------------------------------------------ e2e (host)
    e2 = E2ERound(torch, D, model, codec, stream, so, args.e2e_chunks, xfer=args.e2e_xfer)
    n_host = min(K, 8) + 1
    hosts = [torch.empty(e2.lay.total, dtype=torch.float32, pin_memory=True) for _ in range(n_host)]
    for i, h in enumerate(hosts):
        data.next_round()
        h.copy_(data.x[0])
    torch.cuda.synchronize()
    for i in range(1 + Wm):
        e2.step(hosts[i % n_host], count_payload=(i == Wm))
    e2e_ms = []
    for j in range(K):
        h = hosts[(1 + Wm + j) % n_host]
        D.barrier()
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2.step(h)
        e1.record(stream)
        e1.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    pbytes = e2.payload
    e2e_xfer = e2.xfer
    e2.close()
    e2e_step = D.max(sum(e2e_ms)) / K
    e2e_val = world * e2.upd / (e2e_step * 1e-3) / 1e9
    h2d = e2.upd + pbytes            # inputs up; payloads up for the server
    d2h = pbytes + 4 * e2.lay.total  # payloads down; the aggregate down
    n_e2e_chunks = len(e2.chunks)
    del hosts, e2
    torch.cuda.empty_cache()

    # --------------------------------------------------- nested configs
    nested = {}
    common = 1e-3
    if not args.skip_configs:
        # warm-up rounds: round 0 is direct, the first momentum rounds
        # allocate the state buffers; steady state from the fourth round
        pa = args.aggregate
        nested["federated_64"] = federated_line(torch, D, "resnet50", 64, codec, min(K, 5), 4, flush, so, stream,
                                                common, peer=pa)
        nested["gpt2_medium_16"] = federated_line(torch, D, "gpt2-medium", 16, "q8", min(K, 3), 3, flush, so,
                                                  stream, 0.0, peer=pa)
    if world == 1 and not args.skip_configs:
        nested["resnet18"] = closed_loop_line(torch, D, "resnet18", codec, K, Wm, flush, so, stream)
        nested["int4"] = closed_loop_line(torch, D, "resnet50", "int4", K, Wm, flush, so, stream)
        nested["microbench_512x512x3x3"] = microbench_line(torch, D, 20, flush, so, stream)
        nested["per_layer_api"] = per_layer_line(torch, so)
        nested["pcie"] = pcie_line(torch, D.dev)
        try:
            nested["reference_gpu_v4"] = reference_v4_line(torch, D.dev)
        except Exception as e:   # the baseline is reported, not required
            nested["reference_gpu_v4"] = {"error": str(e)[:300]}
    out = None
    if D.rank == 0:
        cpu, cpu8 = None, None
        if world == 1 and not args.skip_cpu_baseline and ref_library():
            threads = os.cpu_count() or 1
            cpu = cpu_baseline_entry(model, threads, args.cpu_budget_s)
            cpu8 = cpu_baseline_entry(model, 8, args.cpu_budget_s)
        ab_gpu = {"bound": "hbm"}
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": Wm, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded AR(1) Gaussian updates rho=0.9, sigma=1e-3/sqrt(fan_in), ResNet-50 "
                    "state-dict shapes, generated on the GPU)",
            "config": {"workload": f"{model} closed loop, one client per GPU: compress_batch on the client's "
                                   f"encoder + decompress_batch on a separate server decoder writing the decoded "
                                   f"update into the server aggregate (weight 1/{world}, fused into the "
                                   f"reconstruct kernel, no separate decoded copy)"
                                   + (", the aggregate summed over the GPUs" if world > 1 else
                                      "; at one GPU the aggregate is the decoded update itself"),
                       "elements_per_client": fr.lay.numel, "update_bytes_per_client": fr.upd,
                       "clients_per_gpu": 1, "codec": codec, "frames": "GPU zstd frames (Raw / RLE blocks)",
                       "l2": "flushed between steps (256 MiB write, then 256 MiB read of a second buffer; "
                             "outside the timed events)",
                       "parallelism": f"clients sharded over {world} GPU(s)" +
                                      (f", aggregate summed by {collective}" if world > 1 else "")},
            "gpu_launches": launches_timed,
            # `value` is the whole job's raw-update rate (all GPUs); per GPU:
            "value_per_gpu": round(value / world, 3),
            "payload_bytes_per_round": payload,
            "codec_ms_per_step_max": round(codec_max, 4),
            "allreduce_ms_rank0": round(statistics.mean(ar), 4) if world > 1 else 0.0,
            "allreduce_split": split,
            "aggregate_collective": collective,
            "aggregate_choice": choice,
            "aggregate_check": check,
            "rounds": first,
            "roofline": roofline,
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "ms_per_step": round(e2e_step, 4),
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "layer_chunks": n_e2e_chunks,
                    "transfers": e2e_xfer,
                    "how": "pinned host inputs, every chunk's upload queued at the start of the step on an "
                           "upload stream; per layer chunk, once its upload is in, compress_batch (payloads to "
                           "host), decompress_batch into the aggregate, (N > 1) its all-reduce, its download on "
                           "a side stream; inputs up and aggregate down by falcom_copy_sm kernels (sm) or "
                           "copy-engine copies (ce), payloads by the codec's own copies"},
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "cpu_baseline_8_threads": cpu8,
        }
        del ab_gpu
        if "pcie" in nested:
            bound = e2e_link_bound(h2d, d2h, nested["pcie"])
            out["e2e"]["link_bound_ms"] = round(bound, 4)
            out["e2e"]["link_bound_frac"] = round(bound / e2e_step, 4)
        out.update(nested)
        print(json.dumps(out))
    D.close()
    return 0


# ------------------------------------------------------------------ replay
def run_replay(args):
    """Closed loop on captured rounds: each file (the replay layout of the
    reference's benchmark_real.c / profile_appfl_hot_rounds.py) is loaded into
    device memory by the native loader, then compressed on an encoder and
    decompressed on a decoder instance through the C ABI, one round per step
    (files in name order, cycled).  Scalar tensors are left out, as FalComC
    keeps them out of the C codec."""
    import glob
    import torch
    from compressor_b200 import build as B
    from compressor_b200 import replay as R
    from compressor_b200.abi import BatchItemC, Codec, NDArrayC

    files = sorted(glob.glob(args.replay))
    if not files:
        raise SystemExit(f"no replay files match {args.replay}")
    torch.cuda.set_device(0)
    if not os.path.exists(B.OUT):
        B.build()
    os.environ.setdefault("FALCOM_LOG_LEVEL", "ERROR")
    stream = torch.cuda.Stream()      # shared by torch's work and the library's
    torch.cuda.set_stream(stream)
    rounds = []
    for f in files:
        r = R.ReplayRound(f, "device", 0, B.OUT)
        keep = [i for i in range(r.n) if r.items[i].gradient.contents.ndim >= 1]
        items = (BatchItemC * len(keep))()
        for j, i in enumerate(keep):
            items[j].layer_name = r.items[i].layer_name
            items[j].gradient = r.items[i].gradient
        nbytes = sum(r.items[i].gradient.contents.total_size * r.dtypes[i].itemsize for i in keep)
        rounds.append((r, items, len(keep), nbytes))
    client = rounds[0][0].client.encode() or b"Client1"
    enc = Codec(B.OUT, client=client.decode())
    dec = Codec(B.OUT, client=client.decode())
    for c in (enc, dec):
        assert c.lib.falcom_set_residual_codec(c.h, args.codec.encode()) == 0
        c.lib.falcom_set_stream(c.h, ctypes.c_void_p(stream.cuda_stream))
    outs = [(ctypes.POINTER(NDArrayC) * n)() for _, _, n, _ in rounds]
    flush = L2Flush(torch, "cuda")

    def one(k):
        _, items, n, nbytes = rounds[k % len(rounds)]
        o = outs[k % len(rounds)]
        flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        r1 = enc.lib.momentum_compressor_compress_batch(enc.h, items, n, client)
        r2 = dec.lib.momentum_compressor_decompress_batch(dec.h, items, n, client, o)
        e1.record(stream)
        e1.synchronize()
        if r1 != 0 or r2 != 0:
            raise RuntimeError(f"codec failed on {files[k % len(files)]}: {r1} {r2}")
        enc.lib.falcom_free_batch(items, n, o)
        return e0.elapsed_time(e1), nbytes

    for k in range(args.warmup):
        one(k)
    ms, tot = [], 0
    for k in range(args.warmup, args.warmup + args.steps):
        t, nb = one(k)
        ms.append(t)
        tot += nb
    total_ms = sum(ms)
    print(json.dumps({
        "metric": "replay closed-loop codec ms/round; raw-update GB/s", "value": round(tot / (total_ms * 1e-3) / 1e9, 3),
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": f"replay files {args.replay} ({len(files)} rounds)",
        "config": {"workload": "captured rounds, compress_batch + decompress_batch on device-resident tensors",
                   "codec": args.codec, "client": client.decode(),
                   "l2": "flushed between steps (256 MiB write, then 256 MiB read of a second buffer; outside the timed events)"}}))
    enc.close()
    dec.close()
    for r, _, _, _ in rounds:
        r.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="resnet50")
    ap.add_argument("--codec", default="q8", choices=["q8", "int4", "raw"])
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-configs", action="store_true",
                    help="headline step only (no federated / GPT-2 / per-config lines)")
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--aggregate", default="auto", choices=["auto", "peer", "oneshot", "synced", "nccl"],
                    help="N > 1: how the server aggregate is summed over the GPUs (peer: reduce-scatter fused "
                         "into the decoder over NVLink + shard sum / all-gather kernel; oneshot: local "
                         "aggregates, then one in-place all-reduce kernel over NVLink peer memory between two "
                         "NCCL barriers; synced: the same kernel with its barriers on peer flags; nccl: "
                         "all-reduce; auto: the fastest in untimed trial rounds whose FedAvg check passes)")
    ap.add_argument("--e2e-chunks", type=int, default=3,
                    help="layer chunks of the pipelined host-buffer step (e2e)")
    ap.add_argument("--e2e-xfer", default="sm", choices=list(E2ERound.XFER),
                    help="e2e bulk transfers: sm = falcom_copy_sm kernels, ce = copy-engine copies, lib = inputs "
                         "uploaded inside compress_batch")
    ap.add_argument("--mode", default="full", choices=["full", "value"],
                    help="value: only the device-resident timed loop (for profiler runs)")
    ap.add_argument("--replay", default=None,
                    help="glob of captured replay rounds (.bin): time the closed loop on them instead")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        return run_reference(args)
    if args.replay:
        return run_replay(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

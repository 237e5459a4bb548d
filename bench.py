#!/usr/bin/env python
"""Benchmark of the B200 FalCom codec on the ResNet-50 closed loop.

One step = one hot round of one client's ResNet-50 update (266 tensors,
23,573,952 fp32): momentum_compressor_compress_batch on the client's encoder
instance followed by momentum_compressor_decompress_batch on a separate
server-side decoder instance, through the C ABI.  Residual codec q8.

  value    raw-update GB/s over all ranks (update bytes / device time of the
           step, max over ranks), inputs resident in HBM, payloads and
           decoded outputs in device memory
  e2e      the same round with host buffers: pinned host inputs, payloads
           returned to host memory, decoded outputs in host memory, so the
           host<->device copies are inside the timed step
  roofline dominant kernel: algorithmic bytes per launch / mean launch time
           (CUDA events on the library's stream), against the measured HBM
           copy bandwidth
  cpu_baseline  the reference's own grouped OpenMP codec (built from its
           sources, SZ3 stubbed) on the same workload on this host's cores

Multi-GPU (torchrun): every rank runs its own client (weak scaling, no data
collective); device times are reduced with MAX over ranks.
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
        "enc_pass1_stats_sign": 246_334_464,
        "enc_pass2_variance": 193_776_128,
        "enc_pass3_predict": 342_665_216,
        "enc_pass4_quantize_pack": 201_771_776,
        "dec_prefix": 259_840,
        "dec_reconstruct": 438_323_456,
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


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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
            # a short timed region can end before the first sample: wait for
            # one more sample (taken as the region ends) before stopping
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
                "reasons": sorted(reasons), "samples": len(sm)}


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
    from compressor_b200.abi import Codec, HostArray
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
            from compressor_b200.abi import BatchItemC, NDArrayC
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
                         "sample": f"{len(times)} full closed-loop rounds after {args.warmup} warm-up rounds"},
        "e2e": {"value": round(gbs, 5), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))
    return 0


# ------------------------------------------------------------------- ours
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


def make_rounds_on_device(torch, model: str, n_rounds: int, seed: int, device):
    """AR(1) Gaussian updates (rho 0.9, sigma 1e-3/sqrt(fan_in)) generated on
    the GPU with a seeded generator, packed in the flat layout."""
    from compressor_b200 import workloads as W
    lay = W.Layout.of(model)
    sigma = torch.zeros(lay.total, device=device)
    for o, s in zip(lay.offsets, lay.shapes):
        n = int(np.prod(s))
        sigma[o:o + n] = 1e-3 / float(np.sqrt(W.fan_in(s)))
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = []
    state = None
    for _ in range(n_rounds):
        noise = torch.randn(lay.total, device=device, generator=g) * sigma
        state = noise if state is None else 0.9 * state + noise
        out.append(state.clone())
    return lay, out


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from compressor_b200 import build as B
    from compressor_b200.abi import Codec, PreparedBatch, kernel_times
    if not os.path.exists(B.OUT):
        B.build()
    os.environ.setdefault("FALCOM_LOG_LEVEL", "ERROR")

    model = args.model
    K, Wm = args.steps, args.warmup
    n_rounds = 1 + Wm + K
    lay, rounds = make_rounds_on_device(torch, model, n_rounds, seed=1000 + rank, device=dev)
    offs_b = [4 * o for o in lay.offsets]
    upd = lay.numel * 4
    stream = torch.cuda.current_stream()

    def new_pair():
        enc = Codec(B.OUT, client=f"Client{rank + 1}")
        dec = Codec(B.OUT, client=f"Client{rank + 1}")
        for c in (enc, dec):
            assert c.lib.falcom_set_residual_codec(c.h, args.codec.encode()) == 0
            c.lib.falcom_set_stream(c.h, ctypes.c_void_p(stream.cuda_stream))
        return enc, dec

    client = f"Client{rank + 1}".encode()
    flush = L2Flush(torch, dev)

    def closed_loop(enc, dec, pb, base_ptr, count, e0=None, e1=None):
        """One round through the C ABI; e0/e1 (CUDA events on the library's
        stream) bracket exactly the two codec calls."""
        pb.set_pointers(base_ptr, offs_b)
        if e0 is not None:
            e0.record(stream)
        r1 = pb.compress(enc.h, client)
        r2 = pb.decompress(dec.h, client)
        if e1 is not None:
            e1.record(stream)
        if r1 != 0 or r2 != 0:
            raise RuntimeError(f"codec failed: {r1} {r2} {enc.lib.falcom_last_error(enc.h)} "
                               f"{dec.lib.falcom_last_error(dec.h)}")
        nbytes = pb.payload_bytes()
        launches = enc.lib.falcom_last_launches(enc.h) + dec.lib.falcom_last_launches(dec.h)
        pb.release()
        count[0] += launches
        return nbytes

    # ------------------------------------------------ device-resident value
    enc, dec = new_pair()
    pb = PreparedBatch(enc.lib, lay.names, lay.shapes)
    cnt = [0]
    closed_loop(enc, dec, pb, rounds[0].data_ptr(), cnt)          # round 0: direct
    for t in range(1, 1 + Wm):
        closed_loop(enc, dec, pb, rounds[t].data_ptr(), cnt)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms = []
    cnt = [0]
    payload = 0
    with ClockSampler(local) as clk:
        for t in range(1 + Wm, n_rounds):
            flush()                             # L2 flush outside the timed events
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            payload = closed_loop(enc, dec, pb, rounds[t].data_ptr(), cnt, e0, e1)
            e1.synchronize()
            step_ms.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    tot = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms = float(tot.item())
    ms_per_step = total_ms / K
    value = world * upd / (ms_per_step * 1e-3) / 1e9
    launches_timed = cnt[0]

    if args.mode == "value":
        enc.close()
        dec.close()
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
                              "steps": K, "warmup": Wm, "ms_per_step": round(ms_per_step, 4),
                              "mode": "value-only (profiler run)"}))
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # ------------------------------------------------- per-kernel roofline
    enc.lib.falcom_set_kernel_timing(enc.h, 1)
    dec.lib.falcom_set_kernel_timing(dec.h, 1)
    for t in range(1 + Wm, n_rounds):
        flush()
        closed_loop(enc, dec, pb, rounds[t].data_ptr(), [0])
    kt = kernel_times(enc.lib, enc.h)
    kd = kernel_times(dec.lib, dec.h)
    ktimes = {k: (v[0] + kd[k][0], v[1] + kd[k][1]) for k, v in kt.items()}
    enc.close()
    dec.close()

    from compressor_b200 import workloads as Wl
    ab = Wl.algorithmic_bytes(model, args.codec)
    q = {"q8": 1.0, "int4": 0.5, "raw": 4.0}[args.codec]
    me, de = ab["momentum_elements"], ab["direct_elements"]
    # algorithmic bytes per launch of each kernel (all kernels predicted):
    alg = {
        "enc_pass1_stats_sign": me * 12 + de * 8,          # read cur, prev; write history copy
        "enc_pass2_variance": me * 8,                       # read cur, prev
        "enc_pass3_predict": me * 16,                       # read cur, prev, mem; write mem
        "enc_pass4_quantize_pack": me * (8 + q) + de * (4 + q),   # read cur, mem; write codes
        "dec_reconstruct": me * (20 + q) + de * (8 + q),    # read q, prev, mem; write mem, history, output
        "dec_prefix": ab["kernels"] / 8,
        "frames_write": ab["kernels"] / 8 * 2 * 2,
        "frames_expand": ab["kernels"] / 8 * 2 * 2,
    }
    shares = {k: v[0] for k, v in ktimes.items() if v[1] > 0}
    dom = max(shares, key=shares.get)
    avg_ms = ktimes[dom][0] / ktimes[dom][1]
    achieved = alg[dom] / (avg_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "traffic": NCU_TRAFFIC.get((model, args.codec), {}).get(dom),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one steady-state launch",
                "algorithmic_bytes_per_launch": int(alg[dom]), "avg_launch_ms": round(avg_ms, 5),
                "kernel_share": {k: round(v / sum(shares.values()), 4) for k, v in shares.items()},
                "kernel_ms_per_round": {k: round(v[0] / K, 5) for k, v in ktimes.items() if v[1] > 0},
                "launches_per_round": {k: round(v[1] / K, 2) for k, v in ktimes.items() if v[1] > 0},
                "closed_loop_algorithmic_bytes": int(ab["bytes_per_round"]),
                "closed_loop_frac": round(ab["bytes_per_round"] / (ms_per_step * 1e-3) / 1e9 / peak, 4)}

    # ------------------------------------------------------------ e2e (host)
    enc2, dec2 = new_pair()
    pb2 = PreparedBatch(enc2.lib, lay.names, lay.shapes)
    hosts = [torch.empty(lay.total, dtype=torch.float32, pin_memory=True) for _ in range(min(K, 8) + 1 + Wm)]
    for i, h in enumerate(hosts):
        h.copy_(rounds[min(i, n_rounds - 1)])
    torch.cuda.synchronize()
    for i in range(1 + Wm):
        closed_loop(enc2, dec2, pb2, hosts[i].data_ptr(), [0])
    e2e_ms = []
    h2d = d2h = 0
    for j in range(K):
        h = hosts[1 + Wm + j % (len(hosts) - 1 - Wm)]
        flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        pbytes = closed_loop(enc2, dec2, pb2, h.data_ptr(), [0], e0, e1)
        e1.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
        h2d = upd + pbytes          # inputs up; payloads up for the decoder
        d2h = pbytes + upd          # payloads down; decoded update down
    enc2.close()
    dec2.close()
    e2e_t = torch.tensor([sum(e2e_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms_step = float(e2e_t.item()) / K
    e2e_val = world * upd / (e2e_ms_step * 1e-3) / 1e9

    out = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.skip_cpu_baseline and ref_library():
            threads = os.cpu_count() or 1
            ct = cpu_reference_loop(model, 20, 1, threads, budget_s=args.cpu_budget_s)
            cms = 1e3 * statistics.mean(ct)
            cpu = {"value": round(upd / (cms * 1e-3) / 1e9, 5), "unit": "GB/s", "cores": threads,
                   "kind": "reference", "ms_per_round": round(cms, 2),
                   "sample": f"{len(ct)} full ResNet-50 closed-loop rounds (compress_batch + decompress_batch) "
                             f"of the reference grouped OpenMP build, SZ3 stubbed, after 1 warm-up round"}
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": Wm, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded AR(1) Gaussian updates rho=0.9, sigma=1e-3/sqrt(fan_in), "
                    "ResNet-50 state-dict shapes)",
            "config": {"workload": f"{model} single-client closed loop per GPU: compress_batch + "
                                   f"decompress_batch of 266 tensors through the C ABI, separate "
                                   f"encoder/decoder instances, residual codec {args.codec}, GPU zstd frames",
                       "elements_per_client": lay.numel, "update_bytes_per_client": upd,
                       "clients_per_gpu": 1, "codec": args.codec,
                       "l2": "flushed between steps (256 MiB write, then 256 MiB read of a second buffer; outside the timed events)",
                       "parallelism": f"replicas x{world} (independent clients)"},
            "gpu_launches": launches_timed,
            "payload_bytes_per_round": payload,
            "roofline": roofline,
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "ms_per_step": round(e2e_ms_step, 4),
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------- federated
def run_federated(args):
    """Federated round per step: every rank compresses its clients' updates
    (one encoder instance per client) and decodes them on one server decoder
    instance whose weighted aggregate is fused into the decode, then the sum
    all-reduce of the aggregate over NCCL.  With --ar-chunks C > 1 the round
    runs in C layer chunks and each chunk's all-reduce is issued as soon as
    that chunk is decoded, overlapping the later chunks' codec work."""
    import torch
    import torch.distributed as dist
    from compressor_b200 import build as B
    from compressor_b200 import federated as F
    from compressor_b200 import workloads as W
    from compressor_b200.abi import Codec, PreparedBatch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if not os.path.exists(B.OUT):
        B.build()
    os.environ.setdefault("FALCOM_LOG_LEVEL", "ERROR")
    model = args.model
    K, Wm = args.steps, args.warmup
    lay = W.Layout.of(model)
    n_clients = args.clients_per_gpu * world
    mine = list(F.shard(n_clients, world, rank))
    weights = F.uniform_weights(n_clients)
    upd = lay.numel * 4
    offs_b = [4 * o for o in lay.offsets]
    stream = torch.cuda.current_stream()
    # layer chunks of the pipelined all-reduce (one chunk on a single GPU:
    # nothing to overlap)
    chunks = F.layer_chunks([int(np.prod(s)) for s in lay.shapes], args.ar_chunks if world > 1 else 1)
    agg_layout = F.AggregateLayout(list(lay.names), [tuple(s) for s in lay.shapes], list(lay.offsets), lay.total)
    chunk_offs_b = [offs_b[i0:i1] for i0, i1 in chunks]
    chunk_c_offs = [(ctypes.c_size_t * (i1 - i0))(*lay.offsets[i0:i1]) for i0, i1 in chunks]

    def prepared(lib):
        return [PreparedBatch(lib, list(lay.names[i0:i1]), list(lay.shapes[i0:i1])) for i0, i1 in chunks]

    # per-client AR(1) rho 0.9 (own seed) plus a common N(0, 1e-3^2) component
    # drawn once per round with the same seed on every rank
    sigma = torch.zeros(lay.total, device=dev)
    for o, sh in zip(lay.offsets, lay.shapes):
        sigma[o:o + int(np.prod(sh))] = 1e-3 / float(np.sqrt(W.fan_in(sh)))
    gens = []
    for c in mine:
        g = torch.Generator(device=dev)
        g.manual_seed(50_000 + c)
        gens.append(g)
    gcom = torch.Generator(device=dev)
    gcom.manual_seed(49_999)
    states = [None] * len(mine)
    xs = [torch.empty(lay.total, device=dev) for _ in mine]

    def next_round():
        common = torch.randn(lay.total, device=dev, generator=gcom) * 1e-3
        for j in range(len(mine)):
            noise = torch.randn(lay.total, device=dev, generator=gens[j]) * sigma
            states[j] = noise if states[j] is None else states[j].mul_(0.9).add_(noise)
            torch.add(states[j], common, out=xs[j])

    def new_instances():
        encs = [Codec(B.OUT, client=f"Client{c + 1}") for c in mine]
        dec = Codec(B.OUT, client="server")
        for c in encs + [dec]:
            assert c.lib.falcom_set_residual_codec(c.h, args.codec.encode()) == 0
            c.lib.falcom_set_stream(c.h, ctypes.c_void_p(stream.cuda_stream))
        return encs, dec

    agg = torch.zeros(lay.total, dtype=torch.float32, device=dev)
    flush = L2Flush(torch, dev)
    cids = [f"Client{c + 1}".encode() for c in mine]

    def fed_step(encs, dec, pbs, ptrs, count, e0=None, ear=None, e1=None):
        if e0 is not None:
            e0.record(stream)
        # the first client's decode stores its weighted update (store mode of
        # the fused aggregate), so the aggregate needs no clearing; the
        # padding between tensors is never written and stays zero
        if not mine:
            agg.zero_()
        ar = F.ChunkedAllreduce(agg, agg_layout, chunks, dist)
        payload = 0
        for g, (i0, i1) in enumerate(chunks):
            pb = pbs[g]
            for j, c in enumerate(mine):
                pb.set_pointers(ptrs[j], chunk_offs_b[g])
                r1 = pb.compress(encs[j].h, cids[j])
                F.set_client_weight(dec.lib, dec.h, agg.data_ptr(), chunk_c_offs[g], i1 - i0, weights[c])
                F.set_aggregate_store(dec.lib, dec.h, j == 0)
                r2 = pb.decompress(dec.h, cids[j])
                if r1 != 0 or r2 != 0:
                    raise RuntimeError(f"codec failed on rank {rank} client {c}: {r1} {r2}")
                payload += pb.payload_bytes()
                count[0] += encs[j].lib.falcom_last_launches(encs[j].h) + dec.lib.falcom_last_launches(dec.h)
                pb.release()
            if ear is not None and g == len(chunks) - 1:
                ear.record(stream)
            ar.chunk_done(g)
        ar.wait()
        if e1 is not None:
            e1.record(stream)
        return payload

    # ------------------------------------------------ device-resident value
    encs, dec = new_instances()
    pbs = prepared(encs[0].lib)
    for _ in range(1 + Wm):
        next_round()
        fed_step(encs, dec, pbs, [x.data_ptr() for x in xs], [0])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    step_ms, ar_ms, cnt, payload = [], [], [0], 0
    with ClockSampler(local) as clk:
        for _ in range(K):
            next_round()
            flush()
            e0, ear, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            payload = fed_step(encs, dec, pbs, [x.data_ptr() for x in xs], cnt, e0, ear, e1)
            e1.synchronize()
            step_ms.append(e0.elapsed_time(e1))
            ar_ms.append(ear.elapsed_time(e1))
    torch.cuda.synchronize()
    tot = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    ms_per_step = float(tot.item()) / K
    value = n_clients * upd / (ms_per_step * 1e-3) / 1e9
    for c in encs + [dec]:
        c.close()

    # ------------------------------------------------------------ e2e (host)
    encs, dec = new_instances()
    pbs = prepared(encs[0].lib)
    hosts = [torch.empty(lay.total, dtype=torch.float32, pin_memory=True) for _ in mine]
    agg_host = torch.empty(lay.total, dtype=torch.float32, pin_memory=True)
    e2e_ms, h2d, d2h = [], 0, 0
    for it in range(1 + Wm + K):
        next_round()
        for h, x in zip(hosts, xs):
            h.copy_(x)
        torch.cuda.synchronize()
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pbytes = fed_step(encs, dec, pbs, [h.data_ptr() for h in hosts], [0], e0)
        agg_host.copy_(agg, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        if it >= 1 + Wm:
            e2e_ms.append(e0.elapsed_time(e1))
            h2d = len(mine) * upd + pbytes       # inputs up, payloads up for the decoder
            d2h = pbytes + len(mine) * upd + 4 * lay.total   # payloads and decoded outputs down, aggregate
    for c in encs + [dec]:
        c.close()
    e2e_t = torch.tensor([sum(e2e_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_step = float(e2e_t.item()) / K
    e2e_val = n_clients * upd / (e2e_step * 1e-3) / 1e9

    if rank == 0:
        peak, peak_kind = measured_peak()
        ab = W.algorithmic_bytes(model, args.codec)
        # per client: the closed loop's bytes plus the fused aggregate (read
        # the decoded tensor, read and write the aggregate: 12 B / element;
        # the first client stores without reading the aggregate: 8 B)
        alg = len(mine) * (ab["bytes_per_round"] + 12 * lay.numel) - (4 * lay.numel if mine else 0)
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": K,
            "warmup": Wm, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (per-client seeded AR(1) Gaussian updates rho=0.9, sigma=1e-3/sqrt(fan_in), "
                    "plus a shared N(0, 1e-3^2) component per round; ResNet-50 state-dict shapes)",
            "config": {"workload": f"federated round of {n_clients} {model} clients, {args.clients_per_gpu} per "
                                   f"GPU: compress_batch per client, decompress_batch on one server decoder "
                                   f"per GPU with the weighted aggregate fused in, NCCL sum all-reduce of "
                                   f"the {lay.numel}-element aggregate in {len(chunks)} layer chunk(s), each "
                                   f"issued once decoded; residual codec {args.codec}",
                       "clients": n_clients, "clients_per_gpu": args.clients_per_gpu,
                       "allreduce_chunks": len(chunks),
                       "elements_per_client": lay.numel, "update_bytes_per_client": upd, "codec": args.codec,
                       "l2": "flushed between steps (256 MiB write, then 256 MiB read of a second buffer; outside the timed events)",
                       "parallelism": f"clients sharded over {world} GPU(s), NCCL all-reduce of the aggregate"},
            "gpu_launches": cnt[0],
            "payload_bytes_per_step_rank0": payload,
            # all-reduce time left after the last chunk's decode (the rest overlaps the codec)
            "allreduce_exposed_ms_rank0": round(statistics.mean(ar_ms), 4),
            "roofline": {"bound": "hbm", "kernel": "federated step (all codec kernels + aggregate)",
                         "achieved": round(alg / (ms_per_step * 1e-3) / 1e9, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(alg / (ms_per_step * 1e-3) / 1e9 / peak, 4), "traffic": None,
                         "algorithmic_bytes_per_step_per_gpu": int(alg)},
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "ms_per_step": round(e2e_step, 4),
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "clocks": clk.summary(),
            "cpu_baseline": None,
        }
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
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
    stream = torch.cuda.current_stream()
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
    ap.add_argument("--cpu-budget-s", type=float, default=20.0)
    ap.add_argument("--mode", default="full", choices=["full", "value"],
                    help="value: only the device-resident timed loop (for profiler runs)")
    ap.add_argument("--federated", action="store_true",
                    help="federated round (decode + weighted aggregate + all-reduce) also on one GPU")
    ap.add_argument("--ar-chunks", type=int, default=1,
                    help="federated round on N > 1 GPUs: layer chunks of the pipelined aggregate all-reduce "
                         "(1 = one all-reduce after the whole decode; more chunks measured slower on B200)")
    ap.add_argument("--clients-per-gpu", type=int, default=1,
                    help="federated round: clients per GPU (64 / N for the 64-client round)")
    ap.add_argument("--replay", default=None,
                    help="glob of captured replay rounds (.bin): time the closed loop on them instead")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        return run_reference(args)
    if args.replay:
        return run_replay(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 or args.federated:
        return run_federated(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

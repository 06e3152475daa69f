#!/usr/bin/env python
"""Benchmark: int8 inferences/sec of the psp-ml inference path on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg4]
                    [--impl ours|reference] [--batch B] [--point B,K]
                    [--no-extras] [--no-e2e] [--no-cpu-baseline]

One process per GPU (torchrun for N > 1).  Default workload: config 4 =
config 3's depthwise-separable network ([96,512,1] int8 input, 3337 logits)
over a global batch of 262144 sharded in contiguous slices across the ranks
(strong scaling, no collective on the data path).  A step is one forward of
the rank's whole slice, micro-batched on the device.

value    inferences/s of the whole job with inputs resident in HBM, from CUDA
         events around K steps, max over ranks.
e2e      the same through pspml_forward with pinned host buffers: every step
         copies its inputs in and its logits out; K steps between barriers,
         max over ranks.
roofline the dominant kernel's algorithmic bytes (or ops) per launch over its
         event-timed duration inside the timed region.
cpu_baseline  the CPU oracle (int8 TFLite semantics, OpenMP) on a bounded
         sample, rank 0 at N=1 only.
configs  (N = 1) the other benchmark configurations, each measured on its own
         in the same run: config 0 (small CNN, batch 65536), config 2 (deep
         CNN, batch 8192) and the nine points of config 1's FC sweep, each
         with inferences/s, a per-layer roofline table and a CPU-oracle rate.

--impl reference times the reference's CPU path on the host cores instead
(the reference is Rust with no int8 kernels and cannot be built here, so its
int8 semantics run as the C oracle port) and prints the same line.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "psp-ml_b200"))
sys.path.insert(0, str(ROOT))

from pspml import capi, netspec, shard  # noqa: E402

METRIC = "int8 inferences/sec"
UNIT = "inferences/s"

# Config 1: one FullyConnected [B,K] x [K,K]^T per point.
CFG1_POINTS = [(b, k) for b in (1, 256, 16384) for k in (512, 2048, 8192)]

WORKLOADS = {
    # name: (config network, batch, batch kind, micro-batch)
    "cfg4": dict(cfg=3, batch=262144, kind="global", micro=8192,
                 desc="config 4: config-3 depthwise-separable CNN, [96,512,1] int8 -> 3337 "
                      "logits, global batch 262144 sharded over the GPUs"),
    "cfg3": dict(cfg=3, batch=2048, kind="per_gpu", micro=2048,
                 desc="config 3: depthwise-separable CNN, batch 2048 per GPU"),
    "cfg2": dict(cfg=2, batch=8192, kind="per_gpu", micro=8192,
                 desc="config 2: 64x64x3 4-stage CNN, batch 8192 per GPU"),
    "cfg1": dict(cfg=1, batch=16384, kind="per_gpu", micro=16384,
                 desc="config 1: one int8 FullyConnected [B,K] x [K,K]^T, input zp -3, "
                      "output zp 5 + ReLU"),
    "cfg0": dict(cfg=0, batch=65536, kind="per_gpu", micro=65536,
                 desc="config 0: 28x28x1 small CNN, batch 65536 per GPU"),
}

# Working sets below this are flushed from L2 (126 MB) before every step.
L2_FLUSH_BYTES = 256 << 20


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), 2.0 * float(d["bf16_tflops"]), "measured"
    return 6650.0, 2.0 * 1590.0, "fallback"


def build_net(cfg: int, point=None):
    if cfg == 1:
        b, k = point
        return netspec.build_fc_sweep(b, k)
    return netspec.BUILDERS[cfg]()


# ------------------------------------------------------------ layer model
def layer_model(net, fused=None):
    """Per-sample algorithmic bytes and ops of every kernel launch (weights
    per launch).  `fused[i] == 1` marks op i as running op i+1 in the same
    kernel: the pair is one entry ("<op>+pw") whose bytes are op i's input
    and op i+1's output (the intermediate stays on chip); op i+1 then has
    no launch of its own."""
    out = []
    fused = fused or [0] * len(net.layers)
    for i, l in enumerate(net.layers):
        ie = int(np.prod(l.in_shape))
        oe = int(np.prod(l.out_shape))
        alias = l.kind == capi.OP_RESHAPE
        out.append(dict(name=l.name, kind=int(l.kind), bytes_per_sample=0 if alias else ie + oe,
                        weight_bytes=l.weight_bytes, ops_per_sample=2 * l.macs_per_sample,
                        launches_per_chunk=0 if alias else 1,
                        tensor=l.kind in (capi.OP_CONV2D, capi.OP_FULLY_CONNECTED)))
    for i, l in enumerate(net.layers):
        if fused[i] == 1 and i + 1 < len(net.layers):
            nxt = net.layers[i + 1]
            a, b = out[i], out[i + 1]
            suffix = "pool" if nxt.kind == capi.OP_MAX_POOL2D else "pw"
            a["name"] = f"{l.name}+{suffix}"
            a["bytes_per_sample"] = int(np.prod(l.in_shape)) + int(np.prod(nxt.out_shape))
            a["weight_bytes"] += b["weight_bytes"]
            a["ops_per_sample"] += b["ops_per_sample"]
            a["tensor"] = a["tensor"] or b["tensor"] or nxt.kind == capi.OP_CONV2D
            b["launches_per_chunk"] = 0
            b["bytes_per_sample"] = 0
            b["ops_per_sample"] = 0
    return out


def layer_table(ops, op_ms, steps, chunks, n_local):
    """Per-launch roofline of every op from its event-timed milliseconds
    (summed over `steps` steps of `chunks` micro-batches each)."""
    hbm_gbs, int8_tops, _ = peaks()
    ridge = int8_tops * 1e12 / (hbm_gbs * 1e9)
    layers = []
    for o, ms in zip(ops, op_ms):
        if o["launches_per_chunk"] == 0:
            continue
        launches = steps * chunks
        avg_ms = max(ms / launches, 1e-6)
        per_launch_samples = n_local / chunks
        byts = o["bytes_per_sample"] * per_launch_samples + o["weight_bytes"]
        flops = o["ops_per_sample"] * per_launch_samples
        gbs = byts / (avg_ms * 1e-3) / 1e9
        tops = flops / (avg_ms * 1e-3) / 1e12
        tensor_bound = o["tensor"] and flops / max(byts, 1) > ridge
        t_roof = max(flops / (int8_tops * 1e12), byts / (hbm_gbs * 1e9))
        layers.append(dict(name=o["name"], ms_per_step=round(ms / steps, 4),
                           share=None, bound="tensor" if tensor_bound else "hbm",
                           gbs=round(gbs, 1), tops=round(tops, 2),
                           frac=round(t_roof / (avg_ms * 1e-3), 4),
                           bytes_per_launch=int(byts), ops_per_launch=int(flops),
                           avg_launch_ms=round(avg_ms, 4)))
    tot = sum(l["ms_per_step"] for l in layers) or 1.0
    for l in layers:
        l["share"] = round(l["ms_per_step"] / tot, 4)
    return layers


def roofline_of(layer, traffic=None):
    """The roofline object of one layer-table entry."""
    hbm_gbs, int8_tops, peak_src = peaks()
    if layer["bound"] == "tensor":
        roof = {"bound": "tensor", "achieved": layer["tops"], "peak": round(int8_tops, 1),
                "unit": "TOPS", "frac": round(layer["tops"] / int8_tops, 4), "traffic": traffic}
    else:
        roof = {"bound": "hbm", "achieved": layer["gbs"], "peak": hbm_gbs, "unit": "GB/s",
                "frac": round(layer["gbs"] / hbm_gbs, 4), "traffic": traffic}
    roof["kernel"] = layer["name"]
    roof["peak_source"] = (f"{peak_src}: HBM = MEASURED_PEAKS hbm_gbs; int8 tensor = 2 x "
                           "bf16_tflops (no int8 measurement)")
    return roof


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="pspml_clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------ CPU oracle
def oracle_rate(net, descs, blob, target_s=15.0, probe=4, max_n=4096):
    """Oracle inferences/s on all host cores over a bounded sample."""
    from oracle import oracle as orc
    threads = host_threads()
    # The probe keeps every thread busy (OpenMP splits the batch), so its
    # rate predicts the sample's and the sample lasts about target_s.
    probe = min(max(probe, 2 * threads), max_n)
    x = net.make_input(probe, tag="cpu-probe")
    t0 = time.perf_counter()
    orc.net_forward_s8(descs, blob, x, threads=threads)
    dt = max(time.perf_counter() - t0, 1e-6)
    n = int(min(max_n, max(probe, target_s * probe / dt)))
    x = net.make_input(n, tag="cpu-sample")
    t0 = time.perf_counter()
    orc.net_forward_s8(descs, blob, x, threads=threads)
    dt = time.perf_counter() - t0
    return n / dt, n, dt


def host_threads():
    """Host cores this process may use (passed explicitly to the oracle:
    torchrun sets OMP_NUM_THREADS=1 for its workers)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def parse_point(s):
    b, k = (int(v) for v in s.split(","))
    if (b, k) not in CFG1_POINTS:
        raise SystemExit(f"--point {s}: not one of config 1's points {CFG1_POINTS}")
    return b, k


# ------------------------------------------------------------- reference arm
def run_reference(args, wl, rank, world):
    if rank != 0:
        return
    point = parse_point(args.point) if wl["cfg"] == 1 else None
    net = build_net(wl["cfg"], point or (256, 2048))
    descs, blob = net.descs_and_blob()
    from oracle import oracle as orc
    orc.lib()
    budget = 150.0 / max(1, args.warmup + args.steps)
    rate0, _, _ = oracle_rate(net, descs, blob, target_s=min(5.0, budget), probe=4)
    n = int(max(4, min(2048, rate0 * min(budget, 20.0))))
    x = net.make_input(n, tag="reference-arm")
    threads = host_threads()
    for _ in range(args.warmup):
        orc.net_forward_s8(descs, blob, x[: max(1, n // 8)], threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        orc.net_forward_s8(descs, blob, x, threads=threads)
        times.append(time.perf_counter() - t0)
    ms = 1000.0 * statistics.mean(times)
    value = n / (ms / 1000.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong" if wl["kind"] == "global" else "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": args.workload, "description": wl["desc"],
                   "samples_per_step": n},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads,
                         "kind": "port",
                         "sample": f"{n} samples of the {args.workload} network per step; the "
                                   "reference (Rust, f32-only kernels) cannot be built here, "
                                   "so its path runs as the C oracle port of TFLite int8 "
                                   "semantics, OpenMP over the batch"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if point is not None:
        line["config"]["point"] = {"B": point[0], "K": point[1]}
    emit(line)


# ------------------------------------------------------------------ our arm
def device_input(net, n, dev, seed):
    """Seeded synthetic inputs generated on the device with the network's
    input distribution (as Network.make_input), resident in HBM."""
    import torch
    in_e = net.in_elems
    x = torch.empty(max(1, n) * in_e, dtype=torch.int8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    chunk = max(1, (1 << 27) // in_e)
    for b0 in range(0, n, chunk):
        b1 = min(n, b0 + chunk)
        m = (b1 - b0) * in_e
        if net.input_kind == "gaussian_spectrogram":
            v = torch.randn(m, generator=gen, device=dev) * 25.0 - 40.0
            v = v.round().clamp_(-128, 127)
        elif net.input_kind == "uniform_int8":
            v = torch.randint(-128, 128, (m,), generator=gen, device=dev).float()
        else:
            v = torch.randint(0, 256, (m,), generator=gen, device=dev).float() - 128.0
        x[b0 * in_e:b1 * in_e] = v.to(torch.int8)
        del v
    return x


def measure_net(ctx, net, n_local, micro, steps, warmup, dev, stream, seed, flush_buf=None):
    """Device-resident forwards of one network: per-op CUDA events over
    `steps` steps (L2 flushed before each when `flush_buf` is given).
    Returns the layer table, the step time (sum of the op times) and the
    rate."""
    import torch
    descs, blob = net.descs_and_blob()
    model = capi.Model(ctx, descs, blob, micro)
    try:
        x_dev = device_input(net, n_local, dev, seed)
        y_dev = torch.empty(max(1, n_local) * net.out_elems, dtype=torch.int8, device=dev)
        for _ in range(warmup):
            model.forward_device(x_dev.data_ptr(), y_dev.data_ptr(), n_local, stream)
        torch.cuda.synchronize()
        ctx.check_device()
        op_ms = np.zeros(len(net.layers))
        for _ in range(steps):
            if flush_buf is not None:
                flush_buf.add_(1)
            op_ms += np.array(model.forward_timed(x_dev.data_ptr(), y_dev.data_ptr(), n_local,
                                                  stream))
        torch.cuda.synchronize()
        ctx.check_device()
        ops = layer_model(net, [model.op_fused(i) for i in range(len(net.layers))])
        chunks = -(-n_local // micro)
        layers = layer_table(ops, op_ms, steps, chunks, n_local)
        ms = float(op_ms.sum()) / steps
        launches = steps * chunks * sum(o["launches_per_chunk"] for o in ops)
        del x_dev, y_dev
    finally:
        model.close()
    return dict(layers=layers, ms_per_step=ms, value=n_local / (ms / 1000.0),
                gpu_launches=int(launches), descs=descs, blob=blob)


def run_extras(args, ctx, dev, stream):
    """Configs 0, 2 and 1 measured on their own (N = 1): inferences/s, the
    per-layer roofline table and the dominant kernel, plus a short CPU-oracle
    rate for each."""
    import torch
    flush = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    steps = max(3, min(args.steps, 5))
    out = {}
    for name in ("cfg0", "cfg2"):
        wl = WORKLOADS[name]
        net = build_net(wl["cfg"])
        r = measure_net(ctx, net, wl["batch"], wl["micro"], steps, 2, dev, stream, seed=99)
        dom = max(r["layers"], key=lambda l: l["ms_per_step"])
        entry = {"value": round(r["value"], 1), "unit": UNIT, "batch": wl["batch"],
                 "micro_batch": wl["micro"], "steps": steps,
                 "ms_per_step": round(r["ms_per_step"], 3), "description": wl["desc"],
                 "l2": "activations larger than L2 (no flush needed)",
                 "roofline": roofline_of(dom), "layers": r["layers"]}
        if not args.no_cpu_baseline:
            rate, n, dt = oracle_rate(net, r["descs"], r["blob"], target_s=3.0)
            entry["cpu_baseline"] = {"value": round(rate, 3), "unit": UNIT,
                                     "cores": host_threads(), "kind": "port",
                                     "sample": f"{n} samples in {dt:.1f} s"}
        out[name] = entry
        torch.cuda.empty_cache()
    points = []
    for b, k in CFG1_POINTS:
        net = build_net(1, (b, k))
        ws = b * k * 2 + k * k
        r = measure_net(ctx, net, b, b, max(steps, 10), 2, dev, stream, seed=7,
                        flush_buf=flush if ws < L2_FLUSH_BYTES else None)
        l = r["layers"][0]
        p = {"B": b, "K": k, "N": k, "value": round(r["value"], 1), "unit": UNIT,
             "ms": round(r["ms_per_step"], 5), "bound": l["bound"], "gbs": l["gbs"],
             "tops": l["tops"], "frac": l["frac"],
             "l2": "L2 flushed before every step" if ws < L2_FLUSH_BYTES else
                   "working set larger than L2"}
        if not args.no_cpu_baseline:
            rate, n, dt = oracle_rate(net, r["descs"], r["blob"], target_s=1.0, probe=4,
                                      max_n=b)
            p["cpu_baseline"] = {"value": round(rate, 3), "unit": UNIT,
                                 "cores": host_threads(), "kind": "port",
                                 "sample": f"{n} rows in {dt:.2f} s"}
        points.append(p)
        torch.cuda.empty_cache()
    out["cfg1"] = {"description": WORKLOADS["cfg1"]["desc"], "points": points}
    del flush
    return out


def run_ours(args, wl, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    point = parse_point(args.point) if wl["cfg"] == 1 else None
    net = build_net(wl["cfg"], point)
    descs, blob = net.descs_and_blob()
    if wl["cfg"] == 1:
        start, stop = 0, point[0]
        global_batch = point[0] * world
    elif wl["kind"] == "global":
        start, stop = shard.slice_for(args.batch or wl["batch"], world, rank)
        global_batch = args.batch or wl["batch"]
    else:
        start, stop = 0, args.batch or wl["batch"]
        global_batch = (args.batch or wl["batch"]) * world
    n_local = stop - start
    micro = min(args.micro or (n_local if wl["cfg"] == 1 else wl["micro"]), max(1, n_local))

    ctx = capi.Context(local_rank)
    ctx.set_timeout_ms(600_000)
    model = capi.Model(ctx, descs, blob, micro)
    stream = torch.cuda.current_stream().cuda_stream

    in_e, out_e = net.in_elems, net.out_elems
    x_dev = device_input(net, n_local, dev, 1234 + rank)
    y_dev = torch.empty(max(1, n_local) * out_e, dtype=torch.int8, device=dev)
    ws = n_local * (in_e + out_e) + blob.nbytes
    flush = (torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
             if ws < L2_FLUSH_BYTES else None)
    torch.cuda.synchronize()

    ops = layer_model(net, [model.op_fused(i) for i in range(len(net.layers))])
    n_ops = len(ops)
    chunks = -(-n_local // micro)

    for _ in range(args.warmup):
        model.forward_device(x_dev.data_ptr(), y_dev.data_ptr(), n_local, stream)
    torch.cuda.synchronize()
    ctx.check_device()

    # ---- timed region: K steps, per-op CUDA events on the launching stream.
    # A working set smaller than L2 is flushed (one 256 MB write) before
    # every step; the step time is then the sum of the op times, which
    # leaves the flush out.
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    op_ms = np.zeros(n_ops)
    ev0.record()
    for _ in range(args.steps):
        if flush is not None:
            flush.add_(1)
        op_ms += np.array(model.forward_timed(x_dev.data_ptr(), y_dev.data_ptr(), n_local,
                                              stream))
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ctx.check_device()
    local_ms = (float(op_ms.sum()) if flush is not None else ev0.elapsed_time(ev1)) / args.steps
    step_ms = max_over_ranks(local_ms)
    value = global_batch / (step_ms / 1000.0)
    gpu_launches = args.steps * chunks * sum(o["launches_per_chunk"] for o in ops)

    # ---- roofline of the dominant kernel (largest share of the timed region)
    layers = layer_table(ops, op_ms, args.steps, chunks, n_local)
    dom = max(layers, key=lambda l: l["ms_per_step"])
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        try:
            t = json.loads(tf.read_text())
            per_sample = t.get(args.workload, {}).get(dom["name"])
            if per_sample is not None:
                traffic = int(per_sample * n_local / chunks)
        except Exception:
            traffic = None
    roof = roofline_of(dom, traffic)

    # ---- end to end: pinned host buffers through pspml_forward, the same
    # K steps between barriers, max over ranks.
    e2e = None
    if not args.no_e2e:
        hin = torch.empty(max(1, n_local) * in_e, dtype=torch.int8).pin_memory()
        hout = torch.empty(max(1, n_local) * out_e, dtype=torch.int8).pin_memory()
        hin.copy_(x_dev)
        torch.cuda.synchronize()
        model.forward(hin.data_ptr(), hout.data_ptr(), n_local)  # warm the pipeline
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            model.forward(hin.data_ptr(), hout.data_ptr(), n_local)
        local_s = (time.perf_counter() - t0) / args.steps
        barrier()
        e2e_s = max_over_ranks(local_s)
        h2d_b = int(n_local * in_e)
        e2e = {"value": round(global_batch / e2e_s, 1), "unit": UNIT,
               "h2d_bytes_per_step": h2d_b, "d2h_bytes_per_step": int(n_local * out_e),
               "steps": args.steps,
               "h2d_gbs_all_ranks": round(h2d_b * world / e2e_s / 1e9, 2)}
        del hin, hout

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as orc
        orc.lib()
        rate, n, dt = oracle_rate(net, descs, blob, max_n=4096 if wl["cfg"] != 1 else n_local)
        cpu = {"value": round(rate, 3), "unit": UNIT, "cores": host_threads(), "kind": "port",
               "sample": f"{n} samples of the {args.workload} network in {dt:.1f} s (C oracle "
                         "of TFLite int8 semantics, OpenMP over the batch)"}

    model.close()
    flushed = flush is not None
    del x_dev, y_dev, flush
    torch.cuda.empty_cache()

    # ---- the other configurations (N = 1)
    extras = None
    if world == 1 and not args.no_extras:
        extras = run_extras(args, ctx, dev, stream)

    if rank == 0:
        config = {"workload": args.workload, "description": wl["desc"],
                  "global_batch": global_batch, "per_rank_batch": n_local,
                  "micro_batch": micro, "parallelism": f"batch-slice x{world}, no collective",
                  "l2": ("L2 flushed (256 MB write) before every step; step time = sum of "
                         "the op times" if flushed else
                         "inputs larger than L2 (no flush needed)"),
                  "macs_per_inference": net.macs_per_sample()}
        if point is not None:
            config["point"] = {"B": point[0], "K": point[1]}
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
            "higher_is_better": True,
            "scaling": "strong" if wl["kind"] == "global" else "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(gpu_launches),
            "clocks": clocks,
            "layers": layers,
        }
        if extras is not None:
            line["configs"] = extras
        emit(line)
    ctx.close()


_RESULT = None  # the process's original standard output: the JSON line only


def emit(line) -> None:
    out = _RESULT if _RESULT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _RESULT
    # Everything else that reaches standard output (library banners such as
    # NCCL's version line, stray prints) goes to standard error, so that the
    # result line is the only line on standard output.
    sys.stdout.flush()
    _RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="cfg4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--micro", type=int, default=0)
    ap.add_argument("--batch", type=int, default=0,
                    help="batch of the workload (global for cfg4, per GPU otherwise); small "
                         "cases for profiling")
    ap.add_argument("--point", default="16384,8192",
                    help="config 1 point B,K when --workload cfg1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the host-buffer pass (short profiling runs)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the other configurations (short profiling runs)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, wl, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

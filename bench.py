#!/usr/bin/env python
"""Benchmark: int8 inferences/sec of the psp-ml inference path on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg4]
                    [--impl ours|reference]

One process per GPU (torchrun for N > 1).  Default workload: config 4 =
config 3's depthwise-separable network ([96,512,1] int8 input, 3337 logits)
over a global batch of 262144 sharded in contiguous slices across the ranks
(strong scaling, no collective on the data path).  A step is one forward of
the rank's whole slice, micro-batched on the device.

value    inferences/s of the whole job with inputs resident in HBM, from CUDA
         events around K steps, max over ranks.
e2e      the same through pspml_forward with pinned host buffers: every step
         copies its inputs in and its logits out.
roofline the dominant kernel's algorithmic bytes (or ops) per launch over its
         event-timed duration inside the timed region.
cpu_baseline  the CPU oracle (int8 TFLite semantics, OpenMP) on a bounded
         sample, rank 0 at N=1 only.

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

WORKLOADS = {
    # name: (config network, batch, batch kind, micro-batch)
    "cfg4": dict(cfg=3, batch=262144, kind="global", micro=8192,
                 desc="config 4: config-3 depthwise-separable CNN, [96,512,1] int8 -> 3337 "
                      "logits, global batch 262144 sharded over the GPUs"),
    "cfg3": dict(cfg=3, batch=2048, kind="per_gpu", micro=2048,
                 desc="config 3: depthwise-separable CNN, batch 2048 per GPU"),
    "cfg2": dict(cfg=2, batch=8192, kind="per_gpu", micro=8192,
                 desc="config 2: 64x64x3 4-stage CNN, batch 8192 per GPU"),
    "cfg0": dict(cfg=0, batch=65536, kind="per_gpu", micro=65536,
                 desc="config 0: 28x28x1 small CNN, batch 65536 per GPU"),
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), 2.0 * float(d["bf16_tflops"]), "measured"
    return 6650.0, 2.0 * 1590.0, "fallback"


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
            a["name"] = f"{l.name}+pw"
            a["bytes_per_sample"] = int(np.prod(l.in_shape)) + int(np.prod(nxt.out_shape))
            a["weight_bytes"] += b["weight_bytes"]
            a["ops_per_sample"] += b["ops_per_sample"]
            a["tensor"] = True
            b["launches_per_chunk"] = 0
            b["bytes_per_sample"] = 0
            b["ops_per_sample"] = 0
    return out


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
def oracle_rate(net, descs, blob, target_s=15.0, probe=4):
    """Oracle inferences/s on all host cores over a bounded sample."""
    from oracle import oracle as orc
    threads = host_threads()
    # The probe keeps every thread busy (OpenMP splits the batch), so its
    # rate predicts the sample's and the sample lasts about target_s.
    probe = max(probe, 2 * threads)
    x = net.make_input(probe, tag="cpu-probe")
    t0 = time.perf_counter()
    orc.net_forward_s8(descs, blob, x, threads=threads)
    dt = max(time.perf_counter() - t0, 1e-6)
    n = int(min(4096, max(probe, target_s * probe / dt)))
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


# ------------------------------------------------------------- reference arm
def run_reference(args, wl, rank, world):
    if rank != 0:
        return
    net = netspec.BUILDERS[wl["cfg"]]()
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
    emit(line)


# ------------------------------------------------------------------ our arm
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

    net = netspec.BUILDERS[wl["cfg"]]()
    descs, blob = net.descs_and_blob()
    if wl["kind"] == "global":
        start, stop = shard.slice_for(wl["batch"], world, rank)
        global_batch = wl["batch"]
    else:
        start, stop = 0, wl["batch"]
        global_batch = wl["batch"] * world
    n_local = stop - start
    micro = min(args.micro or wl["micro"], max(1, n_local))

    ctx = capi.Context(local_rank)
    ctx.set_timeout_ms(600_000)
    model = capi.Model(ctx, descs, blob, micro)
    stream = torch.cuda.current_stream().cuda_stream

    # Synthetic inputs generated on the device (same distributions as
    # Network.make_input), resident in HBM; far larger than the 126 MB L2.
    in_e, out_e = net.in_elems, net.out_elems
    x_dev = torch.empty(n_local * in_e, dtype=torch.int8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    chunk = 4096
    for b0 in range(0, n_local, chunk):
        b1 = min(n_local, b0 + chunk)
        n = (b1 - b0) * in_e
        if net.input_kind == "gaussian_spectrogram":
            v = torch.randn(n, generator=gen, device=dev) * 25.0 - 40.0
            v = v.round().clamp_(-128, 127)
        else:
            v = torch.randint(0, 256, (n,), generator=gen, device=dev).float() - 128.0
        x_dev[b0 * in_e:b1 * in_e] = v.to(torch.int8)
        del v
    y_dev = torch.empty(max(1, n_local) * out_e, dtype=torch.int8, device=dev)
    torch.cuda.synchronize()

    ops = layer_model(net, [model.op_fused(i) for i in range(len(net.layers))])
    n_ops = len(ops)
    chunks = -(-n_local // micro)

    for _ in range(args.warmup):
        model.forward_device(x_dev.data_ptr(), y_dev.data_ptr(), n_local, stream)
    torch.cuda.synchronize()
    ctx.check_device()

    # ---- timed region: K steps, per-op CUDA events on the launching stream
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
        op_ms += np.array(model.forward_timed(x_dev.data_ptr(), y_dev.data_ptr(), n_local,
                                              stream))
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ctx.check_device()
    step_ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    value = global_batch / (step_ms / 1000.0)
    gpu_launches = args.steps * chunks * sum(o["launches_per_chunk"] for o in ops)

    # ---- roofline of the dominant kernel (largest share of the timed region)
    hbm_gbs, int8_tops, peak_src = peaks()
    layers = []
    for o, ms in zip(ops, op_ms):
        if o["launches_per_chunk"] == 0:
            continue
        launches = args.steps * chunks
        avg_ms = ms / launches
        per_launch_samples = n_local / chunks
        byts = o["bytes_per_sample"] * per_launch_samples + o["weight_bytes"]
        flops = o["ops_per_sample"] * per_launch_samples
        gbs = byts / (avg_ms * 1e-3) / 1e9
        tops = flops / (avg_ms * 1e-3) / 1e12
        ridge = int8_tops * 1e12 / (hbm_gbs * 1e9)
        tensor_bound = o["tensor"] and flops / max(byts, 1) > ridge
        t_roof = max(flops / (int8_tops * 1e12), byts / (hbm_gbs * 1e9))
        layers.append(dict(name=o["name"], ms_per_step=round(ms / args.steps, 4),
                           share=None, bound="tensor" if tensor_bound else "hbm",
                           gbs=round(gbs, 1), tops=round(tops, 2),
                           frac=round(t_roof / (avg_ms * 1e-3), 4),
                           bytes_per_launch=int(byts), ops_per_launch=int(flops),
                           avg_launch_ms=round(avg_ms, 4)))
    tot = sum(l["ms_per_step"] for l in layers) or 1.0
    for l in layers:
        l["share"] = round(l["ms_per_step"] / tot, 4)
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
    if dom["bound"] == "tensor":
        roof = {"bound": "tensor", "achieved": dom["tops"], "peak": round(int8_tops, 1),
                "unit": "TOPS", "frac": round(dom["tops"] / int8_tops, 4), "traffic": traffic}
    else:
        roof = {"bound": "hbm", "achieved": dom["gbs"], "peak": hbm_gbs, "unit": "GB/s",
                "frac": round(dom["gbs"] / hbm_gbs, 4), "traffic": traffic}
    roof["kernel"] = dom["name"]
    roof["peak_source"] = (f"{peak_src}: HBM = MEASURED_PEAKS hbm_gbs; int8 tensor = 2 x "
                           "bf16_tflops (no int8 measurement)")

    # ---- end to end: pinned host buffers through pspml_forward
    e2e = None
    if not args.no_e2e:
        hin = torch.empty(n_local * in_e, dtype=torch.int8).pin_memory()
        hout = torch.empty(max(1, n_local) * out_e, dtype=torch.int8).pin_memory()
        hin.copy_(x_dev)
        torch.cuda.synchronize()
        e2e_steps = max(1, min(args.steps, 3))
        model.forward(hin.data_ptr(), hout.data_ptr(), n_local)  # warm the pipeline
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            model.forward(hin.data_ptr(), hout.data_ptr(), n_local)
        e2e_s = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
        e2e = {"value": round(global_batch / e2e_s, 1), "unit": UNIT,
               "h2d_bytes_per_step": int(n_local * in_e),
               "d2h_bytes_per_step": int(n_local * out_e)}

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as orc
        orc.lib()
        rate, n, dt = oracle_rate(net, descs, blob)
        cpu = {"value": round(rate, 3), "unit": UNIT, "cores": host_threads(), "kind": "port",
               "sample": f"{n} samples of the {args.workload} network in {dt:.1f} s (C oracle "
                         "of TFLite int8 semantics, OpenMP over the batch)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3),
            "higher_is_better": True,
            "scaling": "strong" if wl["kind"] == "global" else "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": args.workload, "description": wl["desc"],
                       "global_batch": global_batch, "per_rank_batch": n_local,
                       "micro_batch": micro, "parallelism": f"batch-slice x{world}, no collective",
                       "l2": "inputs larger than L2 (no flush needed)",
                       "macs_per_inference": net.macs_per_sample()},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(gpu_launches),
            "clocks": clocks,
            "layers": layers,
        }
        emit(line)
    model.close()
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
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the host-buffer pass (short profiling runs)")
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

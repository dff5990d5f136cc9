#!/usr/bin/env python3
"""Benchmark of the katago-rs B200 backend: b18c384nbt forward passes at batch 256 per GPU, evals/s.

One step = one forward pass of the b18c384nbt-shaped net (seeded random-init weights, f16 activations with f32
accumulation) over a batch of 256 synthetic positions per GPU (the reference's bench harness inputs,
crates/katago-nn-burn/examples/bench.rs:27-32: plane 0 = mask, stones at ~30%, globals U(-1, 1)).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Our arm prints one JSON line with `value` (device-resident inputs, CUDA events on the handle's stream, L2 flushed
between timed steps), `e2e` (the same through the C ABI's host path kc_enqueue / kc_wait: pinned-host inputs copied
in and output rows copied back every step), the roofline of the dominant kernel class (the 3x3-conv CTA-pair tcgen05 GEMM)
and a CPU baseline (the CPU oracle, rank 0 at N = 1). Under torchrun each rank drives its own GPU with its own
batch (weak scaling, no collective on the data path); the time is the max over ranks.

`--impl reference` times the reference path on the host CPU cores: the reference's `flex` backend needs cargo and
cannot be built here, so its arithmetic is timed through the CPU restatement in oracle/ (kind "port").
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "katago-rs_b200", "python"))

METRIC = "b18c384nbt evals/s at batch 256 per GPU"


def metric_name(args):
    """The headline metric, or the same metric for another --net / --batch (a parity or exploration run)."""
    if args.net == "b18c384nbt" and args.batch == 256:
        return METRIC
    return f"{args.net} evals/s at batch {args.batch} per GPU"
UNIT = "evals/s"
# DRAM bytes (read + write) per 3x3-convolution GEMM launch at batch 256, from the full ncu capture summarised in
# profiles/gemm_pair_b18c384nbt_batch256.md (mean of the two 3x3 launches captured).
CONV3_DRAM_BYTES_PER_LAUNCH = 75.0e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--net", default="b18c384nbt")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--precision", default="f16", choices=["f16", "bf16", "f32"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def reduce_timing(total_ms, rows_per_rank, steps, dist=None, device=None):
    """(value, max_ms): the timed region's device time as the max over ranks, and all ranks' rows / that time
    (every rank runs the same per-GPU batch: weak scaling)."""
    import torch
    t = torch.tensor([float(total_ms)], dtype=torch.float64, device=device)
    world = 1
    if dist is not None and dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        world = dist.get_world_size()
    max_ms = float(t.item())
    return world * rows_per_rank * steps / (max_ms / 1e3), max_ms


def workload(args, rank):
    from katago_cuda import inputs
    return inputs.synthetic_inputs(args.batch, 0xB200 + rank, (19,))


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["bf16_tflops_sustained"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 10 ms during the timed region, through NVML
    (read-only queries); nvidia-smi at its 200 ms period when NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h): SwPowerCap 0x4, HwSlowdown 0x8, SwThermalSlowdown 0x20,
    # HwThermalSlowdown 0x40
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index, torch_device=None):
        self.gpu = gpu_index
        self.dev = torch_device
        self.proc = None
        self.thread = None
        self.path = os.path.join("/tmp", f"kc_clocks_{os.getpid()}.csv")

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        if self.dev is not None:
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
                return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                pass
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def start(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.samples = []
            self.stop_evt = threading.Event()
            max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)

            def run():
                while not self.stop_evt.is_set():
                    try:
                        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), max_mhz,
                                             nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except Exception:
                        pass
                    self.stop_evt.wait(0.01)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_evt.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            reasons = sorted({nm for _, _, r in self.samples for nm, bit in self.REASON_BITS.items() if r & bit})
            return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                    "sm_max_mhz": max(s[1] for s in self.samples), "reasons": reasons,
                    "samples": len(self.samples), "source": "nvml, 10 ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) != self.gpu:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 200 ms"}


def cpu_baseline(args, seconds, threads=0):
    """The CPU oracle (float32, OpenMP over all host cores) on a bounded sample of the same workload."""
    sys.path.insert(0, REPO)
    from katago_cuda import netgen
    from oracle.oracle import OracleNet
    net = OracleNet(netgen.net_bytes(args.net))
    spatial, glob, meta, _ = workload(args, 0)
    per = 8
    net.forward(spatial[:1], glob[:1])  # warm
    done, t0 = 0, time.perf_counter()
    while True:
        i = done % (args.batch - per + 1)
        net.forward(spatial[i:i + per], glob[i:i + per], threads=threads)
        done += per
        el = time.perf_counter() - t0
        if el >= seconds or el > 30:
            break
    return done / el, done, el


def host_threads():
    """The host threads this process may use (its CPU affinity set). Passed to the oracle's OpenMP explicitly:
    torchrun sets OMP_NUM_THREADS=1 for every rank."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, REPO)
    from katago_cuda import netgen
    from oracle.oracle import OracleNet
    net = OracleNet(netgen.net_bytes(args.net))
    spatial, glob, _, _ = workload(args, 0)
    per = 4
    cores = host_threads()
    for i in range(args.warmup):
        net.forward(spatial[:per], glob[:per], threads=cores)
    times = []
    for i in range(args.steps):
        j = (i * per) % (args.batch - per + 1)
        t0 = time.perf_counter()
        net.forward(spatial[j:j + per], glob[j:j + per], threads=cores)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = per * args.steps / tot
    line = {
        "impl": "reference", "metric": metric_name(args), "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.net} forward, {per} boards per step of the batch-{args.batch} workload "
                               f"(CPU sample)", "net": args.net},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{per} boards x {args.steps} steps of the {args.net} batch-{args.batch} workload; "
                                   "the reference flex backend needs cargo (absent), so its arithmetic runs as the "
                                   "C++ restatement in oracle/ (float32, OpenMP on all host threads)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import numpy as np
    import torch

    import katago_cuda as kc
    from katago_cuda import netgen

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))

    prec = {"f16": kc.PRECISION_F16, "bf16": kc.PRECISION_BF16, "f32": kc.PRECISION_F32}[args.precision]
    model = kc.Model(netgen.net_bytes(args.net))
    ctx = kc.Context(model, gpu_idxs=[local], precision=prec)
    h = kc.Handle(ctx, max_batch=args.batch, gpu_idx=local)
    flops_row, conv3_row = model.flops()

    spatial, glob, meta, _ = workload(args, rank)
    dev = torch.device("cuda", local)
    d_sp = torch.from_numpy(spatial).to(dev)
    d_gl = torch.from_numpy(glob).to(dev)
    d_out = torch.zeros((args.batch, h.row_len), dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(h.stream_ptr(), device=dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # > 126 MB L2

    def step():
        h.enqueue_device(args.batch, d_sp.data_ptr(), d_gl.data_ptr(), 0, d_out.data_ptr())

    def timed(k, profiled):
        """k steps on the handle's stream, each bracketed by CUDA events, L2 flushed before each (untimed)."""
        ev_s = [torch.cuda.Event(enable_timing=True) for _ in range(k)]
        ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(k)]
        if profiled:
            h.set_profiling(True)  # resets the per-class accumulators
        for i in range(k):
            with torch.cuda.stream(stream):
                flush.zero_()
                ev_s[i].record(stream)
            step()
            ev_e[i].record(stream)
        stream.synchronize()
        h.synchronize()
        prof = h.profile() if profiled else None
        return sum(ev_s[i].elapsed_time(ev_e[i]) for i in range(k)), prof

    # warm-up: both CUDA graphs (plain, and with per-launch timing events) are captured here
    h.set_profiling(True)
    for _ in range(max(3, args.warmup)):
        step()
    h.synchronize()
    h.set_profiling(False)
    for _ in range(max(3, args.warmup)):
        step()
    h.synchronize()
    launches_per_step = h.launch_count(args.batch)

    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local, dev)
    clocks.start()
    # headline: the plain graph; then the same K steps again with an event pair around every launch, which gives
    # the per-kernel-class device times (the events cost a few percent, so they stay out of the headline)
    total_ms, _ = timed(args.steps, False)
    prof_ms, prof = timed(args.steps, True)
    h.set_profiling(False)
    clk = clocks.stop()
    if dist:
        dist.barrier()
    value, max_ms = reduce_timing(total_ms, args.batch, args.steps, dist, dev)

    # parity spot check of this run's output rows (no oracle: finite values only)
    out = d_out.cpu().numpy()
    if not np.all(np.isfinite(out)):
        raise RuntimeError("non-finite outputs in the timed run")

    # e2e through the C ABI host path: pinned inputs -> H2D -> forward -> D2H rows, every step
    h.spatial[:args.batch] = spatial
    h.glob[:args.batch] = glob
    for _ in range(max(3, args.warmup)):
        h.enqueue(args.batch)
        h.wait()
    if dist:
        dist.barrier()
    e_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        with torch.cuda.stream(stream):
            flush.zero_()
            e_s[i].record(stream)
        h.enqueue(args.batch)
        e_e[i].record(stream)
        h.wait()
    torch.cuda.synchronize()
    e2e_ms = sum(e_s[i].elapsed_time(e_e[i]) for i in range(args.steps))
    e2e_value, _ = reduce_timing(e2e_ms, args.batch, args.steps, dist, dev)

    if rank == 0:
        burst, sustained, hbm, src = peaks()
        conv_ms, conv_n = prof["conv3x3"]
        achieved = None
        frac = None
        if conv_n:
            flops_per_launch = conv3_row * args.batch * args.steps / conv_n
            achieved = flops_per_launch / (conv_ms / conv_n / 1e3) / 1e12
            frac = achieved / sustained
        other = {k: {"ms_per_step": v[0] / args.steps, "launches_per_step": v[1] / args.steps}
                 for k, v in prof.items()}
        line = {
            "metric": metric_name(args), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.precision, "data": "synthetic",
            "config": {"workload": f"{args.net} forward pass, batch {args.batch} per GPU, {args.precision} "
                                   "activations/f32 accumulation, seeded random-init weights",
                       "net": args.net, "batch_per_gpu": args.batch,
                       "parallelism": f"replicas x{world} (no collective)",
                       "l2": "flushed between timed steps (256 MiB write, outside the timed events)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": sustained, "unit": "TFLOP/s", "frac": frac,
                         "traffic": CONV3_DRAM_BYTES_PER_LAUNCH if args.net == "b18c384nbt" and args.batch == 256
                         else None,
                         "kernel": "gemm_pair_kernel (3x3 conv: CTA-pair tcgen05 implicit GEMM, windowed A)",
                         "peak_kind": f"{src} bf16 sustained"},
            "kernels": other,
            "profiled_ms_per_step": prof_ms / args.steps,
            "flops_per_eval": flops_row,
            "model_tflops": flops_row * value / 1e12,
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": args.batch * (h.n_spatial + h.n_global) * 4,
                    "d2h_bytes_per_step": args.batch * h.row_len * 4 + 4},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu_baseline:
            v, n, el = cpu_baseline(args, args.cpu_seconds, threads=host_threads())
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": host_threads(), "kind": "port",
                                    "sample": f"{n} boards of the batch-{args.batch} workload in {el:.1f} s, "
                                              "CPU oracle float32 (reference arithmetic restated in C++), "
                                              "OpenMP on all host threads"}
        print(json.dumps(line), flush=True)
    h.close()
    if dist:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Benchmark of the katago-rs B200 backend: b18c384nbt forward passes at batch 256 per GPU, evals/s.

One step = one forward pass of the b18c384nbt-shaped net (seeded random-init weights, f16 activations with f32
accumulation) over a batch of 256 synthetic positions per GPU (the reference's bench harness inputs,
crates/katago-nn-burn/examples/bench.rs:27-32: plane 0 = mask, stones at ~30%, globals U(-1, 1)).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Our arm prints one JSON line with `value` (device-resident inputs, CUDA events on the handle's stream, L2 flushed
between timed steps), `e2e` (the same through the C ABI's host path kc_enqueue / kc_wait, timed by the host clock:
pinned-host inputs copied in and every output row copied back each step), the roofline of the dominant kernel class
(the 3x3-conv CTA-pair tcgen05 GEMM) and a CPU baseline (the CPU oracle, rank 0 at N = 1). Under torchrun each rank
drives its own GPU with its own batch (weak scaling, no collective on the data path); the time is the max over
ranks. `--in-process` runs the N GPUs as N handles of one process, one host thread each (katago-rs's own layout:
one NN server thread per GPU), and takes the max over the threads.

`--boards 9,13,19` draws each position's board size from the list (the mixed-board configuration, padded into
19x19 under the on-board mask).

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

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "katago-rs_b200", "python"))

METRIC = "b18c384nbt evals/s at batch 256 per GPU"
UNIT = "evals/s"
# DRAM bytes (read + write) per launch of the 3x3-convolution GEMM, from an ncu capture of this benchmark's own
# kernel (`--metrics dram__bytes_read.sum,dram__bytes_write.sum`): one line per workload, "net batch boards bytes".
TRAFFIC_FILE = os.path.join(REPO, "profiles", "conv3x3_dram_bytes_per_launch.txt")


def metric_name(args):
    """The headline metric, or the same metric for another --net / --batch / --boards (a parity, mixed-board or
    exploration run)."""
    if args.net == "b18c384nbt" and args.batch == 256 and args.boards == "19":
        return METRIC
    on = "" if args.boards == "19" else f" on {args.boards.replace(',', '/')} boards"
    return f"{args.net} evals/s at batch {args.batch} per GPU{on}"


def conv3_traffic(args):
    try:
        for line in open(TRAFFIC_FILE):
            f = line.split()
            if len(f) == 4 and not line.startswith("#") and f[:3] == [args.net, str(args.batch), args.boards]:
                return float(f[3])
    except OSError:
        pass
    return None


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--net", default="b18c384nbt")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--boards", default="19", help="board sizes drawn uniformly per position, e.g. 9,13,19")
    ap.add_argument("--precision", default="f16", choices=["f16", "bf16", "f32"])
    ap.add_argument("--in-process", action="store_true",
                    help="--gpus N handles in this one process, one host thread per GPU (katago-rs's NN server "
                         "threads) instead of one process per GPU under torchrun")
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
    sizes = tuple(int(x) for x in args.boards.split(","))
    return inputs.synthetic_inputs(args.batch, 0xB200 + rank, sizes)


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
    print_line(json.dumps(line))


class Runner:
    """One compute handle on one GPU with its benchmark batch: device-resident copies of the inputs (for `value`),
    the handle's pinned staging buffers (for `e2e`), and the L2 flush buffer."""

    def __init__(self, args, ctx, gpu, seed_rank):
        import torch

        import katago_cuda as kc
        self.args = args
        self.gpu = gpu
        self.dev = torch.device("cuda", gpu)
        self.h = kc.Handle(ctx, max_batch=args.batch, gpu_idx=gpu)
        self.spatial, self.glob, _, _ = workload(args, seed_rank)
        with torch.cuda.device(self.dev):
            self.d_sp = torch.from_numpy(self.spatial).to(self.dev)
            self.d_gl = torch.from_numpy(self.glob).to(self.dev)
            self.d_out = torch.zeros((args.batch, self.h.row_len), dtype=torch.float32, device=self.dev)
            self.stream = torch.cuda.ExternalStream(self.h.stream_ptr(), device=self.dev)
            self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=self.dev)  # > 126 MB L2

    def step(self):
        self.h.enqueue_device(self.args.batch, self.d_sp.data_ptr(), self.d_gl.data_ptr(), 0, self.d_out.data_ptr())

    def _flush(self):
        import torch
        with torch.cuda.device(self.dev), torch.cuda.stream(self.stream):
            self.flush.zero_()

    def warm(self):
        """Both CUDA graphs (plain, and with per-launch timing events) are captured here."""
        n = max(3, self.args.warmup)
        self.h.set_profiling(True)
        for _ in range(n):
            self.step()
            self.h.synchronize()
        self.h.set_profiling(False)
        for _ in range(n):
            self.step()
            self.h.synchronize()
        # e2e staging: each position's planes bit-packed once (the caller's input rows), symmetries drawn per row
        from katago_cuda import api
        b = self.args.batch
        for i in range(b):
            self.h.pk_bits[i] = api.pack_spatial(self.spatial[i])
        self.h.pk_glob[:b] = self.glob
        self.h.pk_sym[:b] = np.random.default_rng(self.gpu).integers(0, 8, size=b)
        self.h.pk_opt[:b] = 0.0
        for _ in range(n):
            self.h.enqueue_packed(b, True)
            self.h.wait_finished()

    def timed(self, k, profiled):
        """k steps on the handle's stream, each bracketed by CUDA events on that stream, L2 flushed before each
        (outside the events). Returns (total ms, per-class profile or None)."""
        import torch
        with torch.cuda.device(self.dev):
            ev_s = [torch.cuda.Event(enable_timing=True) for _ in range(k)]
            ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(k)]
            if profiled:
                self.h.set_profiling(True)  # resets the per-class accumulators
            for i in range(k):
                self._flush()
                ev_s[i].record(self.stream)
                self.h.enqueue_device(self.args.batch, self.d_sp.data_ptr(), self.d_gl.data_ptr(), 0,
                                      self.d_out.data_ptr())
                ev_e[i].record(self.stream)
                self.h.synchronize()
            prof = self.h.profile() if profiled else None
            if profiled:
                self.h.set_profiling(False)
            return sum(ev_s[i].elapsed_time(ev_e[i]) for i in range(k)), prof

    def timed_e2e(self, k):
        """k steps through the C ABI host path, timed by the host clock around kc_enqueue_packed + kc_wait: one
        copy of the pinned bit-packed rows, symmetries and globals to the device, the forward pass with each row's
        symmetry applied on the device, the reference's copy_outputs on the device, and the copy of every row's
        NNOutput fields back, plus the host side of both calls. L2 flushed before each step, outside the timed
        region."""
        import torch
        total = 0.0
        for _ in range(k):
            self._flush()
            with torch.cuda.device(self.dev):
                self.stream.synchronize()
            t0 = time.perf_counter()
            self.h.enqueue_packed(self.args.batch, True)
            rows = self.h.wait_finished()
            total += time.perf_counter() - t0
            if not np.isfinite(rows[0, 0]):
                raise RuntimeError("non-finite output in the e2e run")
        return 1e3 * total

    def check_outputs(self):
        out = self.d_out.cpu().numpy()
        if not np.all(np.isfinite(out)):
            raise RuntimeError("non-finite outputs in the timed run")


def run_ours(args):
    import torch

    import katago_cuda as kc
    from katago_cuda import api, netgen

    rank, world, local = dist_env()
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    in_process = args.in_process and world == 1 and args.gpus > 1
    gpus = list(range(args.gpus)) if in_process else [local]
    torch.cuda.set_device(gpus[0])

    prec = {"f16": kc.PRECISION_F16, "bf16": kc.PRECISION_BF16, "f32": kc.PRECISION_F32}[args.precision]
    model = kc.Model(netgen.net_bytes(args.net))
    ctx = kc.Context(model, gpu_idxs=gpus, precision=prec)
    flops_row, conv3_row = model.flops()
    runners = [Runner(args, ctx, g, rank if not in_process else g) for g in gpus]

    def each(fn):
        """fn(runner) on every runner, one host thread per GPU when there are several (katago-rs's NN server
        threads), started together."""
        if len(runners) == 1:
            return [fn(runners[0])]
        import threading
        res = [None] * len(runners)
        err = []
        gate = threading.Barrier(len(runners))

        def go(i):
            try:
                torch.cuda.set_device(runners[i].gpu)
                gate.wait()
                res[i] = fn(runners[i])
            except Exception as e:  # noqa: BLE001
                err.append(e)
        ts = [threading.Thread(target=go, args=(i,)) for i in range(len(runners))]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        if err:
            raise err[0]
        return res

    each(lambda r: r.warm())
    launches_per_step = runners[0].h.launch_count(args.batch)

    if dist:
        dist.barrier()
    for g in gpus:
        torch.cuda.synchronize(g)
    clocks = ClockSampler(gpus[0], torch.device("cuda", gpus[0]))
    clocks.start()
    # headline: the plain graph; then the same K steps again with an event pair around every launch, which gives
    # the per-kernel-class device times (the events cost a few percent, so they stay out of the headline)
    total_ms = max(each(lambda r: r.timed(args.steps, False)[0]))
    profs = each(lambda r: r.timed(args.steps, True))
    prof_ms, prof = profs[0]
    clk = clocks.stop()
    if dist:
        dist.barrier()
    n_units = len(runners)
    value, max_ms = reduce_timing(total_ms, args.batch * n_units, args.steps, dist, runners[0].dev)
    for r in runners:
        r.check_outputs()

    if dist:
        dist.barrier()
    e2e_ms = max(each(lambda r: r.timed_e2e(args.steps)))
    e2e_value, e2e_max_ms = reduce_timing(e2e_ms, args.batch * n_units, args.steps, dist, runners[0].dev)

    if rank == 0:
        burst, sustained, hbm, src = peaks()
        conv_ms, conv_n = prof["conv3x3"]
        achieved = None
        frac = None
        if conv_n:
            flops_per_launch = conv3_row * args.batch * args.steps / conv_n
            achieved = flops_per_launch / (conv_ms / conv_n / 1e3) / 1e12
            frac = achieved / burst
        other = {k: {"ms_per_step": v[0] / args.steps, "launches_per_step": v[1] / args.steps}
                 for k, v in prof.items()}
        h = runners[0].h
        sizes = args.boards.replace(",", "/")
        line = {
            "metric": metric_name(args), "value": value, "unit": UNIT, "n_gpus": world * n_units,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.precision,
            "data": "synthetic",
            "config": {"workload": f"{args.net} forward pass, batch {args.batch} per GPU of {sizes} boards, "
                                   f"{args.precision} activations/f32 accumulation, seeded random-init weights "
                                   "(He-normal / 1/sqrt(fan_in), last layer of each residual branch scaled by "
                                   "1/sqrt(residual adds))",
                       "net": args.net, "batch_per_gpu": args.batch, "boards": sizes,
                       "parallelism": (f"{n_units} handles in one process, one host thread per GPU"
                                       if in_process else f"replicas x{world} (one process per GPU)")
                                      + ", no collective",
                       "l2": "flushed between timed steps (256 MiB write, outside the timed region)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": burst, "unit": "TFLOP/s", "frac": frac,
                         "traffic": conv3_traffic(args),
                         "kernel": "gemm_pair_kernel (3x3 conv: CTA-pair tcgen05 implicit GEMM, windowed A)",
                         "peak_kind": f"{src} bf16 burst (the kernel is timed by its own launch events)"},
            "kernels": other,
            "profiled_ms_per_step": prof_ms / args.steps,
            "flops_per_eval": flops_row,
            "model_tflops": flops_row * value / 1e12,
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": h.pk_bits.ctypes.data - h.pk_sym.ctypes.data + args.batch * h.pk_bits[0].nbytes,
                    "d2h_bytes_per_step": args.batch * api.FINISHED_ROW_LEN * 4 + 4,
                    "ms_per_step": e2e_max_ms / args.steps,
                    "timing": "host clock around kc_enqueue_packed(finish) + kc_wait: bit-packed rows in, device "
                              "symmetry and copy_outputs, NNOutput rows out"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if world == 1 and n_units == 1 and not args.no_cpu_baseline:
            v, n, el = cpu_baseline(args, args.cpu_seconds, threads=host_threads())
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": host_threads(), "kind": "port",
                                    "sample": f"{n} boards of the batch-{args.batch} workload in {el:.1f} s, "
                                              "CPU oracle float32 (reference arithmetic restated in C++, an "
                                              "unoptimised restatement, not the reference's flex backend), "
                                              "OpenMP on all host threads"}
        print_line(json.dumps(line))
    for r in runners:
        r.h.close()
    if dist:
        dist.destroy_process_group()


class StdoutToStderr:
    """Points file descriptor 1 at stderr while the run's libraries may print there (NCCL prints its version banner
    when the first collective builds the communicator), so that stdout carries only the bench's JSON line."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        self.out = os.fdopen(os.dup(self.saved), "w")
        return self

    def emit(self, line):
        self.out.write(line + "\n")
        self.out.flush()

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)
        self.out.close()
        return False


def main():
    args = parse()
    global print_line
    with StdoutToStderr() as guard:
        print_line = guard.emit
        if args.impl == "reference":
            run_reference(args)
        else:
            run_ours(args)


def print_line(line):
    print(line, flush=True)


if __name__ == "__main__":
    main()

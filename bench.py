"""bench.py -- headline benchmark of the B200 quantized-linear library.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kc|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workload (the metric "W4A16 GEMV HBM GB/s"): the
Llama-style 7B decode linear set at batch M = 1 -- per layer the K->N
projections 4096->12288 (QKV), 4096->4096 (O), 4096->22016 (gate+up) and
11008->4096 (down); GPTQ INT4 weights (uniform nibbles, implicit zero-point 8,
group 128, fp16 scales U[0.002, 0.02]); bf16 activations N(0,1); fp32
accumulation and output.  One step = one decode token through a 32-layer
stack: 32 launches (one grouped launch of a layer's four projections each),
3.35 GB of distinct weights per step, so no step reads weights from L2
(126 MB).  value = algorithmic bytes per step / device time per step.

At N > 1 every rank runs the same workload on its own GPU ("replicas only":
a decode GEMV does not shard usefully at M = 1) and value is the aggregate.

The reference arm (--impl reference) times the reference path's CPU
restatement (oracle/, "kind": "port" -- the reference ships no CPU
implementation of this path, only CUDA kernels) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kernel-craft_b200"))

SHAPES = [("qkv", 4096, 12288), ("o", 4096, 4096), ("gate_up", 4096, 22016), ("down", 11008, 4096)]
GROUP = 128
LAYERS = 32
METRIC = "W4A16 GEMV HBM GB/s (7B decode linear set, M=1)"


def layer_bytes(M: int = 1) -> int:
    """Algorithmic bytes of one layer's four GEMVs: packed N*K/2 + fp16 scales
    2*N*K/128 + bf16 x 2*M*K + fp32 y 4*M*N."""
    return sum(N * K // 2 + 2 * N * K // GROUP + 2 * M * K + 4 * M * N for _, K, N in SHAPES)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def profile_traffic() -> dict | None:
    """dram bytes per launch from the committed ncu summary, if one exists."""
    p = ROOT / "profiles" / "gemv_w4a16_layer_traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------
# reference arm: the CPU restatement on the host cores
# --------------------------------------------------------------------------
def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    O.set_num_threads(cores)
    # one step = the four projections of one layer (104.6 MB of weights),
    # a bounded sample of the 32-layer step
    probs = []
    for i, (_, K, N) in enumerate(SHAPES):
        packed, scales = O.make_w4_gptq(N, K, GROUP, seed=10 + i)
        x = O.make_activations_bf16(1, K, seed=20 + i)
        probs.append((packed, scales, x, N, K))

    def step():
        for packed, scales, x, N, K in probs:
            O.gemv_w4a16(packed, scales, x, 1, N, K, GROUP)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    gbs = layer_bytes(1) / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64-accumulate (CPU port)", "data": "synthetic",
        "config": {"workload": "7b-decode-linear-set-m1 (one layer per step on CPU)",
                   "shapes_KN": [[K, N] for _, K, N in SHAPES], "M": 1, "group_size": GROUP},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": "one layer (4 projections, 104.6 MB INT4) per step"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# kc arm
# --------------------------------------------------------------------------
def cpu_baseline_sample() -> dict:
    """The oracle port on the host cores, bounded to ~10-20 s of CPU work."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    O.set_num_threads(cores)
    _, K, N = SHAPES[0]
    packed, scales = O.make_w4_gptq(N, K, GROUP, seed=99)
    x = O.make_activations_bf16(1, K, seed=98)
    O.gemv_w4a16(packed[:64], scales[:64], x, 1, 64, K, GROUP)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        O.gemv_w4a16(packed, scales, x, 1, N, K, GROUP)
        reps += 1
        if time.perf_counter() - t0 > 10.0 or reps >= 50:
            break
    dt = (time.perf_counter() - t0) / reps
    b = N * K // 2 + 2 * N * K // GROUP + 2 * K + 4 * N
    return {"value": round(b / dt / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"QKV projection 4096->12288, M=1, {reps} reps (~10 s)"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kc", choices=["kc", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e pass")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decoder layers per step (default 32; smaller only for profiling)")
    ap.add_argument("--heat-s", type=float, default=1.5,
                    help="seconds of the same workload run right before the timed region "
                         "(the clock sampler covers it and the timed region)")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        run_reference(args)
        return 0

    import torch
    import torch.distributed as dist
    import kc_lib
    from kc_lib import check, lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    dev = torch.device("cuda", torch.cuda.current_device())
    l = lib()
    stream = torch.cuda.current_stream()
    s_ptr = ctypes.c_void_p(stream.cuda_stream)

    # ---- weights: LAYERS distinct layers, resident in HBM -----------------
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    layers = []
    n_layers = args.layers
    for li in range(n_layers):
        probs = []
        for _, K, N in SHAPES:
            packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=gen)
            scales = (torch.rand(N, K // GROUP, device=dev, generator=gen) * 0.018 + 0.002).half()
            x = torch.randn(1, K, device=dev, generator=gen).bfloat16()
            y = torch.empty(1, N, dtype=torch.float32, device=dev)
            probs.append((packed, scales, x, y, N, K))
        arr = (kc_lib.W4A16Problem * 4)(*[
            kc_lib.W4A16Problem(p.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(), N, K)
            for p, s, x, y, N, K in probs])
        layers.append((probs, arr))

    def step():
        for _, arr in layers:
            check(l.kc_gemv_w4a16_grouped(arr, 4, 1, GROUP, s_ptr))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(vis.split(",")[local].strip() if vis else str(local))
    sampler.start()
    t_heat = time.perf_counter()
    while time.perf_counter() - t_heat < args.heat_s:
        for _ in range(10):
            step()
        torch.cuda.synchronize()

    # ---- timed region ------------------------------------------------------
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    bytes_step = layer_bytes(1) * n_layers
    value = world * bytes_step / (ms_step * 1e-3) / 1e9
    per_gpu = bytes_step / (ms_step * 1e-3) / 1e9
    peaks = measured_peaks()

    # ---- e2e: host buffers through the C ABI, copies inside the timed region
    h_x = [[torch.empty_like(x, device="cpu").pin_memory() for _, _, x, _, _, _ in probs]
           for probs, _ in layers]
    h_y = [[torch.empty_like(y, device="cpu").pin_memory() for _, _, _, y, _, _ in probs]
           for probs, _ in layers]
    for li, (probs, _) in enumerate(layers):
        for j, (_, _, x, _, _, _) in enumerate(probs):
            h_x[li][j].copy_(x)
    h2d = sum(x.numel() * x.element_size() for probs, _ in layers for _, _, x, _, _, _ in probs)
    d2h = sum(y.numel() * y.element_size() for probs, _ in layers for _, _, _, y, _, _ in probs)

    def e2e_step():
        if args.no_e2e:
            return
        for li, (probs, arr) in enumerate(layers):
            for j, (_, _, x, _, _, _) in enumerate(probs):
                x.copy_(h_x[li][j], non_blocking=True)
            check(l.kc_gemv_w4a16_grouped(arr, 4, 1, GROUP, s_ptr))
            for j, (_, _, _, y, _, _) in enumerate(probs):
                h_y[li][j].copy_(y, non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    if world > 1:
        dist.barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e3.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3)
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e_val = world * bytes_step / (ms_e2e / args.steps * 1e-3) / 1e9 if not args.no_e2e else None

    traffic = profile_traffic()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample()

    if rank == 0:
        achieved = per_gpu
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded uniform INT4 nibbles, fp16 scales U[0.002,0.02], bf16 N(0,1))",
            "config": {"workload": "7b-decode-linear-set-m1", "layers": n_layers,
                       "shapes_KN": [[K, N] for _, K, N in SHAPES], "M": 1, "group_size": GROUP,
                       "bytes_per_step": bytes_step, "launch": "one grouped launch per layer",
                       "l2": "inputs larger than L2: 32 distinct layers = 3.35 GB per step",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"],
                         "traffic": (traffic or {}).get("dram_bytes_per_launch"),
                         "algorithmic_bytes_per_launch": layer_bytes(1)},
            "cpu_baseline": cpu,
            "e2e": ({"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                     "d2h_bytes_per_step": d2h} if e2e_val is not None else None),
            "gpu_launches": n_layers * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

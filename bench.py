"""bench.py -- benchmarks of the B200 quantized-linear library.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kc|reference]
                    [--workload all|gemv|gemm_w4a16|gemm_fp8|quant_fp8|gemv_int4|mlp_w4a16]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

With no --workload (``all``) one JSON line is printed per workload, in the
order gemv_int4, quant_fp8, gemm_w4a16, gemm_fp8, and last the headline
decode-GEMV line ("W4A16 GEMV HBM GB/s"); the headline is measured first
(after its own heat phase, on a GPU the GEMMs have not heated) and printed
last:

  gemv        the Llama-style 7B decode linear set at batch M = 1 -- per
              layer the K->N projections 4096->12288 (QKV), 4096->4096 (O),
              4096->22016 (gate+up) and 11008->4096 (down); GPTQ INT4 weights
              (uniform nibbles, implicit zero-point 8, group 128, fp16 scales
              U[0.002, 0.02]); bf16 activations N(0,1); fp32 accumulation and
              output; the weights in the library's tile-ordered layout
              (kc_w4a16_tile_weights, converted once at load; --gemv-weights
              packed streams the reference's [N, K/2] layout instead, the
              same bytes).  One step = one decode token through a 32-layer stack:
              32 launches (one grouped launch of a layer's four projections
              each), 3.35 GB of distinct weights per step, so no step reads
              weights from L2 (126 MB).  value = algorithmic bytes per step /
              device time per step.  At N > 1 every GPU runs its own replica
              (a decode GEMV has nothing to exchange at M = 1).
  gemm_w4a16  W4A16 GEMM M=2048, K=8192, N=28672, group 128, bf16 out; at
              N > 1 column parallel (N split, the all-gather fused into the
              GEMM epilogue), strong scaling
  gemm_fp8    FP8 W8A8 GEMM M=4096, K=8192, N=8192, per-token x per-channel
              scales, bf16 out; at N > 1 row parallel (K split, bf16 sum of
              the partials), strong scaling
  quant_fp8   per-token FP8 quantization of fp32 x [8192, 8192] with 1 %
              outlier channels (x20)
  gemv_int4   the reference ABI's fp32 INT4 GEMV, 4096 x 4096
  mlp_w4a16   the reference's MLP block (col-parallel linear -> GELU ->
              row-parallel linear -> all-reduce) on W4A16 weights, M=2048,
              H=4096, I=16384, GELU in the first GEMM's epilogue, fp32 out
              (run with --workload mlp_w4a16)

At N > 1 the sharded GEMMs first pass a correctness gate: the sharded result
on a small problem is compared with the single-GPU kernel's on the same
inputs (bit-equal for the column-parallel GEMM, normwise <= 1e-2 for the
row-parallel one, whose bf16 partials are rounded before the sum); a
mismatch prints an error line for that workload, which is not timed, and
the run ends with exit code 3 after the other workloads.

The reference arm (--impl reference) times the reference path's CPU
restatement (oracle/, "kind": "port" -- the reference ships no CPU
implementation of this path, only CUDA kernels) on the host cores, one
bounded sample of the workload per step, and prints the same sequence of
lines.
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
CPU_SAMPLE_S = 10.0


def layer_bytes(M: int = 1) -> int:
    """Algorithmic bytes of one layer's four GEMVs: packed N*K/2 + fp16 scales
    2*N*K/128 + bf16 x 2*M*K + fp32 y 4*M*N."""
    return sum(N * K // 2 + 2 * N * K // GROUP + 2 * M * K + 4 * M * N for _, K, N in SHAPES)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def profile_traffic(name: str) -> dict | None:
    """DRAM bytes per launch of the workload's dominant kernel, from the
    committed ncu summary (profiles/<kernel>_<workload>.traffic.json)."""
    p = ROOT / "profiles" / f"{name}.traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: str):
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
            # nvidia-smi can take seconds to print its first sample (longer
            # while other ranks start theirs): wait for it, so the heat phase
            # and the timed region that follow are sampled
            t0 = time.perf_counter()
            while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 10.0:
                time.sleep(0.05)
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


def _oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    O.set_num_threads(os.cpu_count() or 1)
    return O


def _timed_sample(fn, budget_s: float = CPU_SAMPLE_S, max_reps: int = 50):
    """Runs fn() until budget_s has passed (at least once); mean seconds per call."""
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        if time.perf_counter() - t0 > budget_s or reps >= max_reps:
            break
    return (time.perf_counter() - t0) / reps, reps


# --------------------------------------------------------------------------
# workloads
# --------------------------------------------------------------------------
class Workload:
    """One benchmark case.  Subclasses fill the device buffers in __init__(),
    launch one step in step() and describe the algorithmic work per step."""
    name = ""
    workload_id = ""       # the config name both arms report
    metric = ""
    unit = "GB/s"
    bound = "hbm"          # or "tensor-bf16" / "tensor-fp8"
    dtype = ""
    data = ""
    launches_per_step = 1
    kernel = ""            # dominant kernel (ncu name)
    profile = ""           # profiles/<profile>.md / .traffic.json

    scaling = "weak"       # "strong" when the ranks split one problem

    def __init__(self, torch, l, dev, s_ptr, rank, world=1):
        self.torch, self.l, self.dev, self.s_ptr, self.rank = torch, l, dev, s_ptr, rank
        self.world = world
        self.gen = torch.Generator(device=dev)
        self.gen.manual_seed(1234 + rank)

    def work_per_step(self) -> float:      # bytes or flops of THIS rank per step
        raise NotImplementedError

    def parallelism(self) -> str:
        return f"replicas x{self.world}"

    def scale(self) -> float:              # work units -> metric units
        return 1e-9 if self.unit == "GB/s" else 1e-12

    def config(self) -> dict:
        raise NotImplementedError

    # e2e: host buffers through the C ABI, copies inside the timed region
    def e2e_prepare(self):
        raise NotImplementedError

    def e2e_step(self):
        raise NotImplementedError

    @staticmethod
    def cpu_sample() -> dict:
        raise NotImplementedError

    @staticmethod
    def reference_step():
        """(fn, work per call in metric units * 1/scale, sample description)"""
        raise NotImplementedError

    def gate(self):
        """Multi-GPU correctness gate, run on every rank before anything is
        timed: (ok, record).  Workloads without an exchange have none."""
        return True, None

    def step_compute_only(self):
        """The step without its collective (None: the workload has none); timed
        apart so the line can name the limiter."""
        return None

    def close(self):
        """Releases what the workload shares with the other ranks."""


def _normwise(a, b) -> float:
    """max |a - b| / max |b| over two tensors (on the device)."""
    d = (a.double() - b.double()).abs().max()
    return float(d / b.double().abs().max().clamp_min(1e-30))


class GemvW4A16(Workload):
    name = "gemv"
    workload_id = "7b-decode-linear-set-m1"
    metric = "W4A16 GEMV HBM GB/s (7B decode linear set, M=1)"
    dtype = "bf16"
    data = "synthetic (seeded uniform INT4 nibbles, fp16 scales U[0.002,0.02], bf16 N(0,1))"
    kernel = "gemv_w4a16"
    profile = "gemv_w4a16_7b_decode_m1"

    def __init__(self, torch, l, dev, s_ptr, rank, world=1, layers=LAYERS, weights="tiled", M=1):
        super().__init__(torch, l, dev, s_ptr, rank, world)
        import kc_lib
        self.kc_lib = kc_lib
        self.weights = weights
        self.M = M
        if M != 1:   # the other batch sizes of the decode configuration
            self.workload_id = f"7b-decode-linear-set-m{M}"
            self.metric = f"W4A16 GEMV HBM GB/s (7B decode linear set, M={M})"
        self.n_layers = layers
        self.launches_per_step = layers
        self.layers = []
        # every activation and every output of a step in one buffer each, so
        # the end-to-end step moves them with one copy in and one copy out
        # (each problem's slice stays 16-byte aligned: K*2 and N*4 bytes)
        kx = sum(K for _, K, _ in SHAPES)
        ny = sum(N for _, _, N in SHAPES)
        self.x_all = torch.randn(layers * kx * M, device=dev, generator=self.gen).bfloat16()
        self.y_all = torch.empty(layers * ny * M, dtype=torch.float32, device=dev)
        xo = yo = 0
        for _ in range(layers):
            probs = []
            for _, K, N in SHAPES:
                packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev,
                                       generator=self.gen)
                scales = (torch.rand(N, K // GROUP, device=dev, generator=self.gen) * 0.018
                          + 0.002).half()
                x = self.x_all[xo:xo + M * K].view(M, K)
                y = self.y_all[yo:yo + M * N].view(M, N)
                xo += M * K
                yo += M * N
                probs.append((packed, scales, x, y, N, K))
            tiled = None
            if self.weights == "tiled":
                # the library's tile-ordered layout, converted once like a
                # checkpoint at load time; the packed copy is dropped
                tiled = []
                for i, (p, sc, x, y, N, K) in enumerate(probs):
                    t = torch.empty(((N + 15) // 16 * 16) * (K // 2), dtype=torch.uint8, device=dev)
                    kc_lib.check(l.kc_w4a16_tile_weights(p.data_ptr(), t.data_ptr(), N, K, s_ptr))
                    tiled.append(t)
                torch.cuda.synchronize()
                probs = [(None, sc, x, y, N, K) for (_, sc, x, y, N, K) in probs]
            arr = (kc_lib.W4A16Problem * 4)(*[
                kc_lib.W4A16Problem(p.data_ptr() if p is not None else None, s.data_ptr(), x.data_ptr(),
                                    y.data_ptr(), N, K)
                for p, s, x, y, N, K in probs])
            tarr = (ctypes.c_void_p * 4)(*[t.data_ptr() for t in tiled]) if tiled else None
            self.layers.append((probs, arr, tiled, tarr))

    use_graph = True      # replay the step's launches as one CUDA graph (--no-graph: eager)

    def _grouped(self, layer, st):
        _, arr, _, tarr = layer
        if tarr is not None:
            self.kc_lib.check(self.l.kc_gemv_w4a16_grouped_tiled(arr, tarr, None, 4, self.M, GROUP, st))
        else:
            self.kc_lib.check(self.l.kc_gemv_w4a16_grouped(arr, 4, self.M, GROUP, st))

    def _launch_all(self):
        # launched on the current stream: the capture stream inside the graph
        # capture, the bench's stream otherwise
        st = ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)
        for layer in self.layers:
            self._grouped(layer, st)

    def _capture(self):
        """The step's 32 grouped launches as one CUDA graph (captured after one
        eager step, which sets the kernel attributes); eager if capture fails."""
        torch = self.torch
        self._launch_all()
        torch.cuda.synchronize()
        try:
            g = torch.cuda.CUDAGraph()
            # thread_local: other threads (e.g. the NCCL watchdog of a
            # multi-rank run) keep their CUDA calls legal during the capture
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._launch_all()
            torch.cuda.synchronize()
            self.graph = g
        except RuntimeError as e:              # fall back, and say so in the config
            self.graph = None
            self.use_graph = False
            self.graph_error = str(e).splitlines()[0][:200]

    def step(self):
        if not self.use_graph:
            self._launch_all()
            return
        if getattr(self, "graph", None) is None:
            self._capture()
            if not self.use_graph:
                return
        self.graph.replay()

    def work_per_step(self):
        return layer_bytes(self.M) * self.n_layers

    def config(self):
        return {"workload": self.workload_id, "layers": self.n_layers,
                "shapes_KN": [[K, N] for _, K, N in SHAPES], "M": self.M, "group_size": GROUP,
                "weights": ("packed [N, K/2] (the reference layout)" if self.weights == "packed" else
                            "tile-ordered (kc_w4a16_tile_weights, converted once at load)"),
                "bytes_per_step": self.work_per_step(),
                "launch": "one grouped launch per layer" + (
                    ", the step's launches replayed as one CUDA graph" if self.use_graph else
                    ", eager" + (f" (graph capture failed: {self.graph_error})"
                                 if hasattr(self, "graph_error") else "")),
                "l2": f"inputs larger than L2: {self.n_layers} distinct layers = "
                      f"{self.work_per_step() / 1e9:.2f} GB per step"}

    E2E_PARTS = 4   # layer groups whose copies overlap the other groups' launches

    def e2e_prepare(self):
        """Host buffers for the end-to-end step, and the step split into
        E2E_PARTS groups of layers, each captured as its own CUDA graph: the
        activations of group i+1 are copied in, and the outputs of group i-1
        copied out, on a copy stream while group i computes."""
        torch = self.torch
        self.h_x = self.x_all.cpu().pin_memory()
        self.h_y = torch.empty(self.y_all.shape, dtype=self.y_all.dtype).pin_memory()
        kx = sum(K for _, K, _ in SHAPES) * self.M
        ny = sum(N for _, _, N in SHAPES) * self.M
        per = (self.n_layers + self.E2E_PARTS - 1) // self.E2E_PARTS
        self.parts = []
        for p0 in range(0, self.n_layers, per):
            p1 = min(self.n_layers, p0 + per)
            self.parts.append((slice(p0 * kx, p1 * kx), slice(p0 * ny, p1 * ny), self.layers[p0:p1]))
        self.copy_stream = torch.cuda.Stream()
        st = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731
        self.part_graphs = []
        for _, _, layers in self.parts:
            for layer in layers:    # one eager pass sets the kernel attributes
                self._grouped(layer, st())
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                for layer in layers:
                    self._grouped(layer, st())
            self.part_graphs.append(g)
        torch.cuda.synchronize()
        return (self.h_x.numel() * self.h_x.element_size(),
                self.h_y.numel() * self.h_y.element_size())

    def e2e_step(self):
        """Every layer's activations in from pinned host memory, the 32
        grouped launches, every output out -- the copies of one layer group
        overlapped with the launches of the others."""
        torch = self.torch
        main, cs = torch.cuda.current_stream(), self.copy_stream
        ev_in = [torch.cuda.Event() for _ in self.parts]
        ev_out = [torch.cuda.Event() for _ in self.parts]
        cs.wait_stream(main)            # the previous step's reads of x are done
        with torch.cuda.stream(cs):
            for i, (xs, _, _) in enumerate(self.parts):
                self.x_all[xs].copy_(self.h_x[xs], non_blocking=True)
                ev_in[i].record(cs)
        for i, (_, ys, _) in enumerate(self.parts):
            main.wait_event(ev_in[i])
            self.part_graphs[i].replay()
            ev_out[i].record(main)
            with torch.cuda.stream(cs):
                cs.wait_event(ev_out[i])
                self.h_y[ys].copy_(self.y_all[ys], non_blocking=True)
        main.wait_stream(cs)            # the step ends when its last output is on the host

    @staticmethod
    def cpu_sample():
        O = _oracle()
        _, K, N = SHAPES[0]
        packed, scales = O.make_w4_gptq(N, K, GROUP, seed=99)
        x = O.make_activations_bf16(1, K, seed=98)
        O.gemv_w4a16(packed[:64], scales[:64], x, 1, 64, K, GROUP)  # warm
        dt, reps = _timed_sample(lambda: O.gemv_w4a16(packed, scales, x, 1, N, K, GROUP))
        b = N * K // 2 + 2 * N * K // GROUP + 2 * K + 4 * N
        return {"value": round(b / dt / 1e9, 3), "unit": "GB/s", "cores": os.cpu_count() or 1,
                "kind": "port", "sample": f"QKV projection 4096->12288, M=1, {reps} reps (~10 s)"}

    @staticmethod
    def reference_step(layers=LAYERS):
        # the kc arm's step: one decode token through 32 layers (--layers as
        # for the kc arm).  The host runs them over two distinct layers' weights
        # in turn (209 MB, more than any host cache, so every layer streams its
        # weights from DRAM as 32 distinct ones would), which keeps the set-up
        # of the weights short on the host
        O = _oracle()
        distinct = []
        for layer in range(min(2, layers)):
            probs = []
            for i, (_, K, N) in enumerate(SHAPES):
                packed, scales = O.make_w4_gptq(N, K, GROUP, seed=1000 + 8 * layer + i)
                x = O.make_activations_bf16(1, K, seed=2000 + 8 * layer + i)
                probs.append((packed, scales, x, N, K))
            distinct.append(probs)

        def fn():
            for layer in range(layers):
                for packed, scales, x, N, K in distinct[layer % len(distinct)]:
                    O.gemv_w4a16(packed, scales, x, 1, N, K, GROUP)
        return fn, layer_bytes(1) * layers, \
            (f"the full step: {layers} layers of 4 projections ({layer_bytes(1) * layers / 1e9:.2f} GB "
             f"INT4 streamed, two distinct layers' weights in turn), M=1")


class GemmW4A16(Workload):
    name = "gemm_w4a16"
    workload_id = "w4a16-gemm-2048x28672x8192"
    metric = "W4A16 GEMM TFLOP/s (M=2048, K=8192, N=28672, group 128)"
    unit = "TFLOP/s"
    bound = "tensor-bf16"
    dtype = "bf16"
    data = "synthetic (seeded uniform INT4 nibbles, fp16 scales U[0.002,0.02], bf16 N(0,1))"
    kernel = "gemm_w4a16"
    profile = "gemm_w4a16_2048x28672x8192"
    M, N, K = 2048, 28672, 8192
    COPIES = 2

    def __init__(self, torch, l, dev, s_ptr, rank, world=1):
        super().__init__(torch, l, dev, s_ptr, rank, world)
        import kc_lib
        self.kc_lib = kc_lib
        M, N, K = self.M, self.N, self.K
        self.n_shard = N // world           # column parallel: this rank's weight rows
        xg = torch.Generator(device=dev)
        xg.manual_seed(77)                  # activations are replicated: same on every rank
        self.sets = []
        for _ in range(self.COPIES):
            x = torch.randn(M, K, device=dev, generator=xg).bfloat16()
            p = torch.randint(0, 256, (self.n_shard, K // 2), dtype=torch.uint8, device=dev,
                              generator=self.gen)
            s = (torch.rand(self.n_shard, K // GROUP, device=dev, generator=self.gen) * 0.018
                 + 0.002).half()
            out = torch.empty(M, N, dtype=torch.bfloat16, device=dev) if world == 1 else None
            self.sets.append((x, p, s, out))
        self.col = None
        if world > 1:
            import tp
            # each output tile leaves the GPU once through the switch's multicast
            # from 4 ranks on (once per peer with the TMA stores); at 2 ranks the
            # multicast would also route the local copy over NVLink
            store = os.environ.get("KC_TP_STORE", "peer" if world == 2 else "nvls")
            try:
                self.col = tp.ColParallelW4A16(M, N, K, GROUP, store=store)
            except RuntimeError:        # no NVLink multicast
                self.col = tp.ColParallelW4A16(M, N, K, GROUP, store="peer")
            self.scaling = "strong"
        self.i = 0

    def step_compute_only(self):
        if self.col is None:
            return None
        x, p, s, _ = self.sets[self.i % self.COPIES]
        if not hasattr(self, "_local"):
            self._local = self.torch.empty(self.M, self.n_shard, dtype=self.torch.bfloat16,
                                           device=self.dev)
        self.kc_lib.check(self.l.kc_gemm_w4a16(x.data_ptr(), p.data_ptr(), s.data_ptr(),
                                               self._local.data_ptr(), 0, self.M, self.n_shard,
                                               self.K, GROUP, self.n_shard, self.s_ptr))
        self.i += 1
        return True

    def _launch(self, x, p, s, out):
        if self.col is not None:   # fused GEMM + all-gather, then a stream barrier
            # back-to-back steps read nothing in between: the previous step's
            # exit barrier already orders the overwrite
            self.col(x, p, s, entry_barrier=False)
            return
        self.kc_lib.check(self.l.kc_gemm_w4a16(x.data_ptr(), p.data_ptr(), s.data_ptr(),
                                               out.data_ptr(), 0, self.M, self.N, self.K, GROUP,
                                               self.N, self.s_ptr))

    def step(self):
        self._launch(*self.sets[self.i % self.COPIES])
        self.i += 1

    def work_per_step(self):
        return 2.0 * self.M * self.n_shard * self.K

    def parallelism(self):
        if self.world == 1:
            return "single GPU"
        how = ("TMA-stored into every GPU's [M, N] buffer by the GEMM epilogue over NVLink"
               if self.col.store == "peer" else
               "written once by the GEMM epilogue through the NVSwitch multicast (multimem.st), "
               "which stores them into every GPU's [M, N] buffer")
        return (f"column parallel x{self.world}: N/{self.world} weight rows per GPU, output tiles "
                f"{how} (fused all-gather), one peer-flag barrier per step")

    def config(self):
        return {"workload": self.workload_id, "M": self.M, "N": self.N, "K": self.K,
                "group_size": GROUP, "out": "bf16",
                "l2": f"{self.COPIES} rotating operand sets, each step also writes the full "
                      "117 MB output (larger than L2)"}

    def _out(self, out):
        return self.col.out if self.col is not None else out

    def e2e_prepare(self):
        x, _, _, out = self.sets[0]
        o = self._out(out)
        self.h_x = x.cpu().pin_memory()
        self.h_out = self.torch.empty(o.shape, dtype=o.dtype).pin_memory()
        return self.h_x.numel() * 2, self.h_out.numel() * 2

    def e2e_step(self):
        x, p, s, out = self.sets[0]
        x.copy_(self.h_x, non_blocking=True)
        self._launch(x, p, s, out)
        self.h_out.copy_(self._out(out), non_blocking=True)

    @classmethod
    def _cpu(cls, rows):
        O = _oracle()
        packed, scales = O.make_w4_gptq(cls.N, cls.K, GROUP, seed=3)
        x = O.make_activations_bf16(rows, cls.K, seed=4)
        return (lambda: O.gemm_w4a16(x, packed, scales, rows, cls.N, cls.K, GROUP)), \
            2.0 * rows * cls.N * cls.K

    @classmethod
    def cpu_sample(cls):
        fn, flops = cls._cpu(8)
        dt, reps = _timed_sample(fn, max_reps=20)
        return {"value": round(flops / dt / 1e12, 5), "unit": "TFLOP/s",
                "cores": os.cpu_count() or 1, "kind": "port",
                "sample": f"8 of 2048 token rows x all 28672 columns, {reps} reps"}

    @classmethod
    def reference_step(cls):
        fn, flops = cls._cpu(8)
        return fn, flops, "8 of 2048 token rows x all 28672 columns per step"

    def gate(self):
        """The column-parallel GEMM with its fused all-gather, on a problem
        every rank builds identically, must equal the single-GPU
        kc_gemm_w4a16 of the full problem bit for bit."""
        if self.world == 1:
            return True, None
        torch = self.torch
        import tp
        M, K, N = 256, 1024, 256 * self.world
        g = torch.Generator(device=self.dev)
        g.manual_seed(4321)
        x = torch.randn(M, K, device=self.dev, generator=g).bfloat16()
        p = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=self.dev, generator=g)
        s = (torch.rand(N, K // GROUP, device=self.dev, generator=g) * 0.018 + 0.002).half()
        ref = torch.empty(M, N, dtype=torch.bfloat16, device=self.dev)
        self.kc_lib.check(self.l.kc_gemm_w4a16(x.data_ptr(), p.data_ptr(), s.data_ptr(),
                                               ref.data_ptr(), 0, M, N, K, GROUP, N, self.s_ptr))
        col = tp.ColParallelW4A16(M, N, K, GROUP, store=self.col.store)
        ps, ss = tp.shard_w4_rows(p, s, self.world, self.rank)
        out = col(x, ps, ss).clone()
        torch.cuda.synchronize()
        col.close()
        ok = bool(torch.equal(out, ref))
        return ok, {"check": f"column parallel x{self.world} ({self.col.store} stores) on "
                             f"[{M}, {K}] x [{N}, {K}]^T vs the single-GPU kc_gemm_w4a16, bit-equal",
                    "passed": ok, "normwise_err": _normwise(out, ref)}

    def close(self):
        if self.col is not None:
            self.col.close()


class GemmFP8(Workload):
    name = "gemm_fp8"
    workload_id = "fp8-w8a8-gemm-4096x8192x8192"
    metric = "FP8 W8A8 GEMM TFLOP/s (M=4096, K=8192, N=8192)"
    unit = "TFLOP/s"
    bound = "tensor-fp8"
    dtype = "e4m3"
    data = ("synthetic (x N(0,1) with 1% outlier channels x20 quantized per token; "
            "W N(0,0.02) quantized per channel)")
    kernel = "gemm_fp8"
    profile = "gemm_fp8_4096x8192x8192"
    M, N, K = 4096, 8192, 8192
    COPIES = 2

    def __init__(self, torch, l, dev, s_ptr, rank, world=1):
        super().__init__(torch, l, dev, s_ptr, rank, world)
        import kc_lib
        self.kc_lib = kc_lib
        M, N, K = self.M, self.N, self.K
        self.k0, self.k1 = rank * K // world, (rank + 1) * K // world  # row parallel: K shard
        self.x32 = self._outlier_x(M, K)
        self.qa_full = torch.empty(M, K, dtype=torch.int8, device=dev)
        self.sets = []
        for _ in range(self.COPIES):
            sa = torch.empty(M, dtype=torch.float32, device=dev)
            kc_lib.check(l.kc_quantize_fp8_per_token(self.x32.data_ptr(), self.qa_full.data_ptr(),
                                                     sa.data_ptr(), M, K, s_ptr))
            w = torch.randn(N, K, device=dev, generator=self.gen) * 0.02
            qw = torch.empty(N, K, dtype=torch.int8, device=dev)
            sw = torch.empty(N, dtype=torch.float32, device=dev)
            kc_lib.check(l.kc_quantize_fp8_per_channel(w.data_ptr(), qw.data_ptr(), sw.data_ptr(),
                                                       N, K, s_ptr))
            del w
            qa = self.qa_full[:, self.k0:self.k1].contiguous()
            qw = qw[:, self.k0:self.k1].contiguous()
            out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            self.sets.append((qa, sa, qw, sw, out))
        self.rp = None
        if world > 1:
            import tp
            # measured (whole-GEMM TFLOP/s; one GPU 2175): the sum fused into
            # the GEMM epilogue 2726 / 2257 / 1980 on 2 / 4 / 8 B200s; NCCL
            # after the GEMM 2018 / 2023 / 1602; the in-switch sum per row
            # block 1771 / 1951 / 1527
            reduce = os.environ.get("KC_TP_REDUCE", "fused")
            kw = dict(chunks=int(os.environ.get("KC_TP_CHUNKS", "4")),
                      comm_sms=int(os.environ.get("KC_TP_COMM_SMS", "16")))
            try:
                self.rp = tp.RowParallelFP8(M, N, reduce=reduce, **kw)
            except RuntimeError:        # no NVLink multicast: NCCL sums under the GEMMs
                self.rp = tp.RowParallelFP8(M, N, reduce="overlap", **kw)
            self.scaling = "strong"
        self.i = 0

    def _outlier_x(self, T, D):
        t = self.torch
        x = t.randn(T, D, device=self.dev, generator=self.gen)
        ch = t.randperm(D, device=self.dev, generator=self.gen)[:max(1, round(0.01 * D))]
        x[:, ch] *= 20.0
        return x

    def step_compute_only(self):
        if self.rp is None:
            return None
        qa, sa, qw, sw, out = self.sets[self.i % self.COPIES]
        self.kc_lib.check(self.l.kc_gemm_fp8(qa.data_ptr(), sa.data_ptr(), qw.data_ptr(),
                                             sw.data_ptr(), out.data_ptr(), 0, self.M, self.N,
                                             self.k1 - self.k0, self.N, self.s_ptr))
        self.i += 1
        return True

    def _launch(self, qa, sa, qw, sw, out):
        if self.rp is not None:   # K-shard partial, then the bf16 sum over NVLink peers
            self.rp(qa, sa, qw, sw, entry_barrier=False)
            return
        self.kc_lib.check(self.l.kc_gemm_fp8(qa.data_ptr(), sa.data_ptr(), qw.data_ptr(),
                                             sw.data_ptr(), out.data_ptr(), 0, self.M, self.N,
                                             self.K, self.N, self.s_ptr))

    def step(self):
        self._launch(*self.sets[self.i % self.COPIES])
        self.i += 1

    def work_per_step(self):
        return 2.0 * self.M * self.N * (self.k1 - self.k0)

    def parallelism(self):
        if self.world == 1:
            return "single GPU"
        how = {"nccl": "an NCCL all-reduce on the same stream",
               "overlap": (f"NCCL all-reduces of {self.rp.chunks} row blocks, each under the next "
                           f"block's GEMM (GEMM on all but {self.rp.comm_sms} SMs)"),
               "peer": ("kc_allreduce_bf16_peer over NVLink peer memory (each GPU reduces 1/N of the "
                        "output in fp32 and writes it to every GPU) between two peer-flag barriers"),
               "fused": ("the GEMM epilogue itself (kc_gemm_fp8_allreduce: each partial tile written "
                         "over NVLink into the receive slot of the rank owning its rows, the owner's "
                         "bf16 sum written into every rank's output), between two peer-flag barriers"),
               "fused_nvls": ("the GEMM epilogue itself with the NVSwitch (kc_gemm_fp8_allreduce_mc: "
                              "each partial tile into this rank's copy of a symmetric buffer, the "
                              "owner's multimem.ld_reduce + multimem.st into every copy), between two "
                              "peer-flag barriers"),
               "nvls": (f"the NVSwitch in place (kc_allreduce_bf16_nvls: multimem.ld_reduce with fp32 "
                        f"accumulation + multimem.st on a symmetric buffer) for {self.rp.chunks} row "
                        f"blocks, each behind a peer-flag barrier and under the next block's GEMM "
                        f"(GEMM on all but {self.rp.comm_sms} SMs)")
               }[self.rp.reduce]
        return (f"row parallel x{self.world}: K/{self.world} code columns per GPU (scales from "
                f"full rows), bf16 partials summed by {how}")

    def config(self):
        return {"workload": self.workload_id, "M": self.M, "N": self.N,
                "K": self.K, "scales": "per-token x per-channel", "out": "bf16",
                "l2": f"{self.COPIES} rotating operand sets of 168 MB (larger than L2)",
                "e2e": "fp32 activations -> kc_quantize_fp8_per_token -> kc_gemm_fp8 -> bf16"}

    def e2e_prepare(self):
        qa, sa, qw, sw, out = self.sets[0]
        self.h_x = self.x32.cpu().pin_memory()
        self.h_out = self.torch.empty(out.shape, dtype=out.dtype).pin_memory()
        return self.h_x.numel() * 4, self.h_out.numel() * 2

    def e2e_step(self):
        qa, sa, qw, sw, out = self.sets[0]
        self.x32.copy_(self.h_x, non_blocking=True)
        self.kc_lib.check(self.l.kc_quantize_fp8_per_token(self.x32.data_ptr(),
                                                           self.qa_full.data_ptr(), sa.data_ptr(),
                                                           self.M, self.K, self.s_ptr))
        if self.world > 1:
            qa.copy_(self.qa_full[:, self.k0:self.k1])
        else:
            qa = self.qa_full
        self._launch(qa, sa, qw, sw, out)
        self.h_out.copy_(self.rp.out if self.rp is not None else out, non_blocking=True)

    @classmethod
    def _cpu(cls, rows):
        O = _oracle()
        x = O.make_outlier_activations(rows, cls.K, seed=1)
        w = O.make_weight_f32(cls.N, cls.K, seed=2)
        qa, sa = O.quantize_fp8_per_token(x)
        qw, sw = O.quantize_fp8_per_token(w)
        return (lambda: O.gemm_fp8_rowcol(qa, sa, qw, sw)), 2.0 * rows * cls.N * cls.K

    @classmethod
    def cpu_sample(cls):
        fn, flops = cls._cpu(16)
        dt, reps = _timed_sample(fn, max_reps=20)
        return {"value": round(flops / dt / 1e12, 5), "unit": "TFLOP/s",
                "cores": os.cpu_count() or 1, "kind": "port",
                "sample": f"16 of 4096 token rows x all 8192 columns, {reps} reps"}

    @classmethod
    def reference_step(cls):
        fn, flops = cls._cpu(16)
        return fn, flops, "16 of 4096 token rows x all 8192 columns per step"

    def gate(self):
        """The row-parallel GEMM and its bf16 sum, on a problem every rank
        builds identically, must match the single-GPU kc_gemm_fp8 of the full
        K (fp32 output) within 1e-2 normwise: each rank's partial is rounded
        to bf16 before the sum."""
        if self.world == 1:
            return True, None
        torch = self.torch
        import tp
        # M: two 128-row tiles per rank (the fused sum owns rows in R blocks)
        M, N, K = 256 * self.world, 512, 512 * self.world
        g = torch.Generator(device=self.dev)
        g.manual_seed(4322)
        x = torch.randn(M, K, device=self.dev, generator=g)
        x[:, torch.randperm(K, device=self.dev, generator=g)[:max(1, K // 100)]] *= 20.0
        w = torch.randn(N, K, device=self.dev, generator=g) * 0.02
        qa = torch.empty(M, K, dtype=torch.int8, device=self.dev)
        qw = torch.empty(N, K, dtype=torch.int8, device=self.dev)
        sa = torch.empty(M, dtype=torch.float32, device=self.dev)
        sw = torch.empty(N, dtype=torch.float32, device=self.dev)
        l, chk = self.l, self.kc_lib.check
        chk(l.kc_quantize_fp8_per_token(x.data_ptr(), qa.data_ptr(), sa.data_ptr(), M, K, self.s_ptr))
        chk(l.kc_quantize_fp8_per_channel(w.data_ptr(), qw.data_ptr(), sw.data_ptr(), N, K, self.s_ptr))
        ref = torch.empty(M, N, dtype=torch.float32, device=self.dev)
        chk(l.kc_gemm_fp8(qa.data_ptr(), sa.data_ptr(), qw.data_ptr(), sw.data_ptr(), ref.data_ptr(),
                          1, M, N, K, N, self.s_ptr))
        k0, k1 = tp.shard_range(K, self.world, self.rank)
        rp = tp.RowParallelFP8(M, N, reduce=self.rp.reduce, chunks=self.rp.chunks, comm_sms=self.rp.comm_sms)
        out = rp(qa[:, k0:k1].contiguous(), sa, qw[:, k0:k1].contiguous(), sw).clone()
        torch.cuda.synchronize()
        rp.close()
        err = _normwise(out, ref)
        ok = err <= 1e-2
        return ok, {"check": f"row parallel x{self.world} ({self.rp.reduce} sum) on "
                             f"[{M}, {K}] x [{N}, {K}]^T vs the single-GPU kc_gemm_fp8, "
                             "normwise <= 1e-2",
                    "passed": ok, "normwise_err": err}

    def close(self):
        if self.rp is not None:
            self.rp.close()


class QuantFP8(Workload):
    name = "quant_fp8"
    workload_id = "fp8-per-token-quant-8192x8192"
    metric = "FP8 E4M3 per-token quantization GB/s (T=8192, D=8192)"
    dtype = "f32->e4m3"
    data = "synthetic (x N(0,1) with 1% of channels, fixed by seed, scaled x20)"
    kernel = "quant_fp8_rows_reg"
    profile = "quant_fp8_rows_8192x8192"
    T, D = 8192, 8192

    def __init__(self, torch, l, dev, s_ptr, rank, world=1):
        super().__init__(torch, l, dev, s_ptr, rank, world)
        import kc_lib
        self.kc_lib = kc_lib
        x = torch.randn(self.T, self.D, device=dev, generator=self.gen)
        ch = torch.randperm(self.D, device=dev, generator=self.gen)[:round(0.01 * self.D)]
        x[:, ch] *= 20.0
        self.x = x
        self.q = torch.empty(self.T, self.D, dtype=torch.int8, device=dev)
        self.s = torch.empty(self.T, dtype=torch.float32, device=dev)

    def step(self):
        self.kc_lib.check(self.l.kc_quantize_fp8_per_token(self.x.data_ptr(), self.q.data_ptr(),
                                                           self.s.data_ptr(), self.T, self.D,
                                                           self.s_ptr))

    def work_per_step(self):
        return self.T * self.D * 4 + self.T * self.D + self.T * 4

    def config(self):
        return {"workload": self.workload_id, "T": self.T, "D": self.D,
                "bytes_per_step": self.work_per_step(),
                "l2": "input 268 MB (larger than L2)"}

    def e2e_prepare(self):
        self.h_x = self.x.cpu().pin_memory()
        self.h_q = self.torch.empty(self.q.shape, dtype=self.q.dtype).pin_memory()
        self.h_s = self.torch.empty(self.s.shape, dtype=self.s.dtype).pin_memory()
        return self.h_x.numel() * 4, self.h_q.numel() + self.h_s.numel() * 4

    def e2e_step(self):
        self.x.copy_(self.h_x, non_blocking=True)
        self.step()
        self.h_q.copy_(self.q, non_blocking=True)
        self.h_s.copy_(self.s, non_blocking=True)

    @classmethod
    def _cpu(cls, rows):
        O = _oracle()
        x = O.make_outlier_activations(rows, cls.D, seed=0)
        return (lambda: O.quantize_fp8_per_token(x)), rows * cls.D * 5 + rows * 4

    @classmethod
    def cpu_sample(cls):
        fn, b = cls._cpu(2048)
        dt, reps = _timed_sample(fn)
        return {"value": round(b / dt / 1e9, 3), "unit": "GB/s", "cores": os.cpu_count() or 1,
                "kind": "port", "sample": f"2048 of 8192 rows, {reps} reps"}

    @classmethod
    def reference_step(cls):
        fn, b = cls._cpu(2048)
        return fn, b, "2048 of 8192 rows per step"


class GemvInt4(Workload):
    name = "gemv_int4"
    workload_id = "int4-gemv-ref-abi-4096x4096"
    metric = "INT4 dequant+GEMV HBM GB/s (reference ABI, fp32, 4096x4096)"
    dtype = "f32"
    data = ("synthetic (uniform nibbles, packed^0x88 with zero points 0, fp32 scales "
            "U[0.002,0.02], fp32 x N(0,1))")
    kernel = "gemv_int4_f32_vec"
    profile = "gemv_int4_f32_4096x4096"
    R = C = 4096
    COPIES = 32   # 32 x 9 MB = 288 MB of distinct weights rotate through L2

    def __init__(self, torch, l, dev, s_ptr, rank, world=1):
        super().__init__(torch, l, dev, s_ptr, rank, world)
        import kc_lib
        self.kc_lib = kc_lib
        R, C = self.R, self.C
        self.sets = []
        for _ in range(self.COPIES):
            p = torch.randint(0, 256, (R, C // 2), dtype=torch.uint8, device=dev, generator=self.gen)
            s = torch.rand(R, C // GROUP, device=dev, generator=self.gen) * 0.018 + 0.002
            z = torch.zeros(R, C // GROUP // 2, dtype=torch.uint8, device=dev)
            self.sets.append((p, s, z))
        self.x = torch.randn(C, device=dev, generator=self.gen)
        self.y = torch.empty(R, dtype=torch.float32, device=dev)
        self.i = 0

    def _launch(self, p, s, z):
        st = ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)
        self.kc_lib.check(self.l.kc_gemv_int4_f32(p.data_ptr(), s.data_ptr(), z.data_ptr(),
                                                  self.x.data_ptr(), self.y.data_ptr(), self.R,
                                                  self.C, GROUP, st))

    # One step = one GEMV over each of the COPIES weight copies, replayed as a
    # CUDA graph: a 9 MB GEMV takes a few microseconds, less than the host
    # needs to issue one launch through ctypes, so eager steps would time the
    # host rather than the kernel.
    launches_per_step = COPIES

    def step(self):
        torch = self.torch
        if getattr(self, "graph", None) is None:
            for args in self.sets:   # one eager pass first
                self._launch(*args)
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
                for args in self.sets:
                    self._launch(*args)
            torch.cuda.synchronize()
        self.graph.replay()

    def work_per_step(self):
        R, C = self.R, self.C
        return self.COPIES * (R * C // 2 + R * (C // GROUP) * 4 + R * (C // GROUP // 2) + C * 4 + R * 4)

    def config(self):
        return {"workload": self.workload_id, "rows": self.R, "cols": self.C,
                "group_size": GROUP, "bytes_per_step": self.work_per_step(),
                "launch": f"{self.COPIES} GEMVs per step (one per weight copy), replayed as one CUDA graph",
                "e2e": "per GEMV: x in from pinned host memory, the launch, y out (no graph)",
                "l2": f"{self.COPIES} rotating weight copies = 288 MB (larger than L2)"}

    def e2e_prepare(self):
        self.h_x = self.x.cpu().pin_memory()
        self.h_y = self.torch.empty(self.y.shape, dtype=self.y.dtype).pin_memory()
        return self.COPIES * self.h_x.numel() * 4, self.COPIES * self.h_y.numel() * 4

    def e2e_step(self):
        # the reference ABI's use: every GEMV with its own copies in and out
        for args in self.sets:
            self.x.copy_(self.h_x, non_blocking=True)
            self._launch(*args)
            self.h_y.copy_(self.y, non_blocking=True)

    @classmethod
    def _cpu(cls):
        O = _oracle()
        rng = np.random.default_rng(0)
        p = rng.integers(0, 256, (cls.R, cls.C // 2), dtype=np.uint8)
        s = rng.uniform(0.002, 0.02, (cls.R, cls.C // GROUP)).astype(np.float32)
        z = np.zeros((cls.R, cls.C // GROUP // 2), np.uint8)
        x = rng.standard_normal(cls.C).astype(np.float32)
        b = cls.R * cls.C // 2 + cls.R * (cls.C // GROUP) * 4 + z.size + cls.C * 4 + cls.R * 4
        return (lambda: O.gemv_int4(p, s, z, x, cls.R, cls.C, GROUP)), b

    @classmethod
    def cpu_sample(cls):
        fn, b = cls._cpu()
        dt, reps = _timed_sample(fn, max_reps=200)
        return {"value": round(b / dt / 1e9, 3), "unit": "GB/s", "cores": os.cpu_count() or 1,
                "kind": "port", "sample": f"config 0 GEMV, {reps} reps"}

    @classmethod
    def reference_step(cls):
        fn, b = cls._cpu()
        return fn, b, "one config-0 GEMV per step"


class MlpW4A16(Workload):
    name = "mlp_w4a16"
    workload_id = "w4a16-mlp-block-2048x4096x16384"
    metric = "W4A16 MLP block TFLOP/s (M=2048, H=4096, I=16384, GELU, group 128)"
    unit = "TFLOP/s"
    bound = "tensor-bf16"
    dtype = "bf16"
    data = "synthetic (seeded uniform INT4 nibbles, fp16 scales U[0.002,0.02], bf16 N(0,1))"
    kernel = "gemm_w4a16"
    profile = "gemm_w4a16_mlp_2048x4096x16384"
    launches_per_step = 2
    M, H, I = 2048, 4096, 16384
    COPIES = 2

    def __init__(self, torch, l, dev, s_ptr, rank, world=1):
        super().__init__(torch, l, dev, s_ptr, rank, world)
        import tp
        M, H, I = self.M, self.H, self.I
        self.i_shard = I // world           # W1 rows / W2 columns of this rank
        xg = torch.Generator(device=dev)
        xg.manual_seed(78)                  # activations are replicated: same on every rank
        self.x = torch.randn(M, H, device=dev, generator=xg).bfloat16()
        self.sets = []
        for _ in range(self.COPIES):
            w1p = torch.randint(0, 256, (self.i_shard, H // 2), dtype=torch.uint8, device=dev,
                                generator=self.gen)
            w1s = (torch.rand(self.i_shard, H // GROUP, device=dev, generator=self.gen) * 0.018
                   + 0.002).half()
            w2p = torch.randint(0, 256, (H, self.i_shard // 2), dtype=torch.uint8, device=dev,
                                generator=self.gen)
            w2s = (torch.rand(H, self.i_shard // GROUP, device=dev, generator=self.gen) * 0.018
                   + 0.002).half()
            self.sets.append((w1p, w1s, w2p, w2s))
        self.blk = tp.MLPBlockW4A16(M, H, I, GROUP)
        if world > 1:
            self.scaling = "strong"
        self.i = 0

    def step(self):
        self.blk(self.x, *self.sets[self.i % self.COPIES])
        self.i += 1

    def work_per_step(self):
        return 4.0 * self.M * self.H * self.i_shard

    def parallelism(self):
        if self.world == 1:
            return "single GPU"
        return (f"tensor parallel x{self.world}: W1 rows and W2 columns I/{self.world} per GPU, "
                "no communication between the GEMMs, one NCCL fp32 all-reduce per step")

    def config(self):
        return {"workload": self.workload_id, "M": self.M, "H": self.H,
                "I": self.I, "group_size": GROUP, "activation": "gelu_quick (x*sigmoid(1.702x))",
                "out": "fp32",
                "l2": f"{self.COPIES} rotating weight sets of 66 MB each, and the 64 MB bf16 "
                      "intermediate written and read per step (larger than L2 together)"}

    def e2e_prepare(self):
        self.h_x = self.x.cpu().pin_memory()
        self.h_y = self.torch.empty(self.blk.y.shape, dtype=self.blk.y.dtype).pin_memory()
        return self.h_x.numel() * 2, self.h_y.numel() * 4

    def e2e_step(self):
        self.x.copy_(self.h_x, non_blocking=True)
        self.blk(self.x, *self.sets[0])
        self.h_y.copy_(self.blk.y, non_blocking=True)

    @classmethod
    def _cpu(cls, rows):
        O = _oracle()
        w1p, w1s = O.make_w4_gptq(cls.I, cls.H, GROUP, seed=40)
        w2p, w2s = O.make_w4_gptq(cls.H, cls.I, GROUP, seed=41)
        x = O.make_activations_bf16(rows, cls.H, seed=42)
        return (lambda: O.mlp_block_w4a16(x, w1p, w1s, w2p, w2s, rows, cls.H, cls.I, GROUP)), \
            4.0 * rows * cls.H * cls.I

    @classmethod
    def cpu_sample(cls):
        fn, flops = cls._cpu(8)
        dt, reps = _timed_sample(fn, max_reps=20)
        return {"value": round(flops / dt / 1e12, 5), "unit": "TFLOP/s",
                "cores": os.cpu_count() or 1, "kind": "port",
                "sample": f"8 of 2048 token rows through the whole block, {reps} reps"}

    @classmethod
    def reference_step(cls):
        fn, flops = cls._cpu(8)
        return fn, flops, "8 of 2048 token rows through the whole block per step"


WORKLOADS = {w.name: w for w in (GemvW4A16, GemmW4A16, GemmFP8, QuantFP8, GemvInt4, MlpW4A16)}
# the default run: one line each, the headline decode GEMV last
DEFAULT_SET = ("gemv_int4", "quant_fp8", "gemm_w4a16", "gemm_fp8", "gemv")
# the headline (gemv) is measured first -- in its own heat phase, not on a GPU
# the GEMMs before it have heated -- and its line is printed last


def _selected(args) -> list:
    return list(DEFAULT_SET) if args.workload == "all" else [args.workload]


def _spread(ms: list) -> dict:
    """Median and 10th / 90th percentiles of per-step device times (ms)."""
    a = np.asarray(ms, np.float64)
    return {"median": round(float(np.median(a)), 4), "p10": round(float(np.percentile(a, 10)), 4),
            "p90": round(float(np.percentile(a, 90)), 4), "n": int(a.size)}


def fp8_peak() -> dict | None:
    """The dense FP8 tensor-core figure measured on this pool's B200s with
    torch._scaled_mm (profiles/fp8_peak.json, written by a builder run)."""
    p = ROOT / "profiles" / "fp8_peak.json"
    if p.exists():
        return json.loads(p.read_text())
    return None


# --------------------------------------------------------------------------
# reference arm: the CPU restatement on the host cores
# --------------------------------------------------------------------------
def run_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    for name in _selected(args):
        W = WORKLOADS[name]
        fn, work, sample = W.reference_step(args.layers) if W is GemvW4A16 else W.reference_step()
        for _ in range(args.warmup):
            fn()
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            fn()
            times.append((time.perf_counter() - t0) * 1e3)
        dt = sum(times) / len(times) / 1e3
        scale = 1e-9 if W.unit == "GB/s" else 1e-12
        val = work / dt * scale
        cores = os.cpu_count() or 1
        line = {
            "impl": "reference", "metric": W.metric, "value": round(val, 5), "unit": W.unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 3), "step_ms": _spread(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "CPU port (f64 accumulation where the path reduces)", "data": "synthetic",
            "config": {"workload": W.workload_id, "sample": sample},
            "cpu_baseline": {"value": round(val, 5), "unit": W.unit, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(val, 5), "unit": W.unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# kc arm
# --------------------------------------------------------------------------
def _max_over_ranks(torch, dist, world, dev, vals):
    if world == 1:
        return list(vals)
    t = torch.tensor(list(vals), device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def run_workload(name, args, torch, dist, l, dev, stream, s_ptr, world, rank, local, held=None) -> int:
    """One workload: gate (N > 1), warm-up, heat, K timed steps, e2e, one
    JSON line from rank 0.  Returns the exit status (3: the gate failed)."""
    W = WORKLOADS[name]
    if W is GemvW4A16:
        wl = W(torch, l, dev, s_ptr, rank, world, layers=args.layers, weights=args.gemv_weights,
               M=args.gemv_m)
        wl.use_graph = not args.no_graph
    else:
        wl = W(torch, l, dev, s_ptr, rank, world)
    torch.cuda.synchronize()

    ok, gate = wl.gate()
    if world > 1:
        t = torch.tensor([1.0 if ok else 0.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok = bool(t.item() == 1.0)
    if not ok:
        if rank == 0:
            print(json.dumps({"metric": wl.metric, "error": "multi-GPU correctness gate failed",
                              "gate": gate, "n_gpus": world}), flush=True)
        wl.close()
        return 3

    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    # heat phase sized from a timing taken after the warm-up (the first
    # warm-up steps include one-time set-up such as a graph capture); a step
    # COUNT every rank agrees on, since steps may contain collectives
    probe = 3
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(probe):
        wl.step()
    p1.record(stream)
    torch.cuda.synchronize()
    per_step = _max_over_ranks(torch, dist, world, dev, [p0.elapsed_time(p1) / probe / 1e3])[0]
    heat_steps = int(min(args.heat_s / max(per_step, 1e-6), 20000))

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(vis.split(",")[local].strip() if vis else str(local))
    sampler.start()
    for i in range(heat_steps):
        wl.step()
        if i % 8 == 7:
            torch.cuda.synchronize()
    torch.cuda.synchronize()

    # ---- timed region: exactly K steps, an event between steps ---------------
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    evs[0].record(stream)
    for i in range(args.steps):
        wl.step()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    ms = evs[0].elapsed_time(evs[-1])
    # max over ranks: the whole region, and each step's time
    both = _max_over_ranks(torch, dist, world, dev, [ms] + step_ms)
    ms, step_ms = both[0], both[1:]
    ms_step = ms / args.steps
    work = wl.work_per_step()
    sc = wl.scale()
    per_gpu = work / (ms_step * 1e-3) * sc
    value = world * per_gpu

    # ---- the step without its collective (sharded GEMMs): names the limiter
    compute_only_ms = None
    if wl.step_compute_only() is not None:
        for _ in range(2):
            wl.step_compute_only()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(args.steps):
            wl.step_compute_only()
        c1.record(stream)
        torch.cuda.synchronize()
        compute_only_ms = _max_over_ranks(torch, dist, world, dev, [c0.elapsed_time(c1) / args.steps])[0]

    # ---- e2e: host buffers through the C ABI, copies inside the timed region
    e2e = None
    if not args.no_e2e:
        h2d, d2h = wl.e2e_prepare()
        for _ in range(2):
            wl.e2e_step()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(args.steps):
            wl.e2e_step()
            stream.synchronize()
        e3.record(stream)
        torch.cuda.synchronize()
        ms_e2e = _max_over_ranks(torch, dist, world, dev, [e2.elapsed_time(e3)])[0]
        e2e = {"value": round(world * work / (ms_e2e / args.steps * 1e-3) * sc, 3),
               "unit": wl.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    peaks = measured_peaks()
    if wl.bound == "hbm":
        peak, unit, bound, psrc = peaks["hbm_gbs"], "GB/s", "hbm", peaks["source"]
    elif wl.bound == "tensor-bf16":
        # the timed GEMMs run after a 1.5 s heat phase under the power cap: the
        # sustained cuBLAS figure is the like-for-like denominator
        peak, unit, bound = peaks["bf16_tflops_sustained"], "TFLOP/s", "tensor"
        psrc = peaks["source"] + " (cuBLAS bf16, sustained under the power cap)"
    else:
        f8 = fp8_peak()
        unit, bound = "TFLOP/s", "tensor"
        if f8 is not None:
            peak = f8["fp8_tflops_sustained"]
            psrc = ("builder-measured dense FP8: torch._scaled_mm e4m3, sustained under the power "
                    "cap (profiles/fp8_peak.json)")
        else:
            peak = 2 * peaks["bf16_tflops_sustained"]
            psrc = peaks["source"] + " (2 x cuBLAS bf16 sustained; no measured fp8 peak)"
    traffic = profile_traffic(wl.profile)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = W.cpu_sample()

    if rank == 0:
        cfg = wl.config()
        cfg["parallelism"] = wl.parallelism()
        if gate is not None:
            cfg["gate"] = gate
        if compute_only_ms is not None:
            cfg["split_ms"] = {"step": round(ms_step, 4), "compute_only": round(compute_only_ms, 4),
                               "collective_exposed": round(ms_step - compute_only_ms, 4)}
        line = {
            "metric": wl.metric, "value": round(value, 3), "unit": wl.unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "step_ms": _spread(step_ms),
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None, "dtype": wl.dtype,
            "data": wl.data, "config": cfg,
            "roofline": {"bound": bound, "achieved": round(per_gpu, 1), "peak": peak,
                         "unit": unit, "frac": round(per_gpu / peak, 4), "peak_source": psrc,
                         "traffic": (traffic or {}).get("dram_bytes_per_launch"),
                         "kernel": wl.kernel,
                         "algorithmic_work_per_launch": work / wl.launches_per_step},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": wl.launches_per_step * args.steps,
            "clocks": clocks,
        }
        if held is not None:
            held.append(json.dumps(line))
        else:
            print(json.dumps(line), flush=True)
    wl.close()
    del wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return 0


def measure_peak(kind: str, seconds: float, reps: int) -> dict:
    """Dense tensor-core throughput of the library GEMM this pool's roofline
    denominators come from: torch.matmul bf16 8192^3 ("bf16") or
    torch._scaled_mm e4m3 x e4m3 -> bf16 8192^3 with unit scales ("fp8");
    best of `reps` CUDA-event timed launches (burst) and the mean over
    `seconds` of back-to-back launches (sustained, under the power cap)."""
    import torch
    n = 8192
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    a = torch.randn(n, n, device=dev, generator=g)
    b = torch.randn(n, n, device=dev, generator=g)
    if kind == "bf16":
        a, b = a.bfloat16(), b.bfloat16()
        fn = lambda: torch.matmul(a, b)  # noqa: E731
    else:
        a8 = a.to(torch.float8_e4m3fn)
        b8 = b.to(torch.float8_e4m3fn).t()     # column-major second operand
        one = torch.ones((), device=dev)
        fn = lambda: torch._scaled_mm(a8, b8, scale_a=one, scale_b=one,  # noqa: E731
                                      out_dtype=torch.bfloat16)
    flops = 2.0 * n ** 3
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    sampler = ClockSampler(str(torch.cuda.current_device()))
    sampler.start()
    count, t0 = 0, time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    while time.perf_counter() - t0 < seconds:
        for _ in range(8):
            fn()
        count += 8
        torch.cuda.synchronize()
    e1.record()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    return {"kind": kind, "gemm": f"{n}^3", "how": ("torch.matmul bf16" if kind == "bf16" else
                                                     "torch._scaled_mm e4m3 x e4m3 -> bf16"),
            f"{kind}_tflops": round(flops / (best * 1e-3) / 1e12, 1),
            f"{kind}_tflops_sustained": round(flops * count / (e0.elapsed_time(e1) * 1e-3) / 1e12, 1),
            "sustained_launches": count, "clocks": clocks, "torch": torch.__version__}


def tc_calibration() -> None:
    """One launch each of cuBLAS bf16 8192^3 (torch.matmul), torch._scaled_mm
    fp8 8192^3 and the library's two tcgen05 GEMMs at configs 3 and 4, inside a
    cudaProfilerStart/Stop window (ncu --profile-from-start off): the same
    tensor-pipe counters on a library GEMM next to ours."""
    import torch
    from kc_lib import check, lib
    l = lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    n = 8192
    a = torch.randn(n, n, device=dev, generator=g).bfloat16()
    b = torch.randn(n, n, device=dev, generator=g).bfloat16()
    a8, b8 = a.float().to(torch.float8_e4m3fn), b.float().to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)
    M, N, K = GemmW4A16.M, GemmW4A16.N, GemmW4A16.K
    x = torch.randn(M, K, device=dev, generator=g).bfloat16()
    p = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g)
    sc = (torch.rand(N, K // GROUP, device=dev, generator=g) * 0.018 + 0.002).half()
    o = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    M4, N4, K4 = GemmFP8.M, GemmFP8.N, GemmFP8.K
    qa = torch.randint(-100, 100, (M4, K4), dtype=torch.int8, device=dev, generator=g)
    qw = torch.randint(-100, 100, (N4, K4), dtype=torch.int8, device=dev, generator=g)
    sa, sw = torch.rand(M4, device=dev, generator=g), torch.rand(N4, device=dev, generator=g)
    o4 = torch.empty(M4, N4, dtype=torch.bfloat16, device=dev)

    def run():
        torch.matmul(a, b)
        torch._scaled_mm(a8, b8, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        check(l.kc_gemm_w4a16(x.data_ptr(), p.data_ptr(), sc.data_ptr(), o.data_ptr(), 0, M, N, K,
                              GROUP, N, st))
        check(l.kc_gemm_fp8(qa.data_ptr(), sa.data_ptr(), qw.data_ptr(), sw.data_ptr(), o4.data_ptr(),
                            0, M4, N4, K4, N4, st))
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    run()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"tc_calibration": "ok"}), flush=True)


def stream_floor(reps: int = 20) -> dict:
    """The floor the config-0 GEMV is measured against: the library's plain
    streaming-read kernel (kc_selftest_stream_read, same CTA shape and loads in
    flight as gemv_int4_f32_vec) over the GEMV's bytes per launch, 32 rotating
    buffers replayed as one CUDA graph exactly like the GemvInt4 step, and the
    same graph of 32 empty launches (the launch floor)."""
    import torch
    from kc_lib import check, lib
    l = lib()
    dev = torch.device("cuda", torch.cuda.current_device())
    R, C = GemvInt4.R, GemvInt4.C
    nbytes = R * C // 2 + R * (C // GROUP) * 4 + R * (C // GROUP // 2) + C * 4 + R * 4
    bufs = [torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=dev)
            for _ in range(GemvInt4.COPIES)]
    sink = torch.zeros(4, dtype=torch.int32, device=dev)
    out = {"bytes_per_launch": nbytes, "launches_per_graph": GemvInt4.COPIES}
    for label, size in (("read", nbytes), ("empty", 0)):
        def launches():
            st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for buf in bufs:
                check(l.kc_selftest_stream_read(buf.data_ptr(), size, 0x9E3779B9, sink.data_ptr(), st))
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            launches()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                launches()
            for _ in range(5):
                g.replay()
            torch.cuda.synchronize()
            times = []
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                g.replay()
                e1.record(s)
                e1.synchronize()
                times.append(e0.elapsed_time(e1) * 1e3 / GemvInt4.COPIES)
        us = float(np.median(times))
        out[f"{label}_us_per_launch"] = round(us, 3)
        if size:
            out["read_gbs"] = round(nbytes / us / 1e3, 1)
        del g
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tc-calibration", action="store_true",
                    help="run cuBLAS bf16/fp8 and the two tcgen05 GEMMs once in a profiler window")
    ap.add_argument("--stream-floor", action="store_true",
                    help="time a plain streaming read of the config-0 GEMV's bytes per launch")
    ap.add_argument("--peak", choices=["bf16", "fp8"], default=None,
                    help="measure a library GEMM's dense tensor-core peak instead (one JSON line)")
    ap.add_argument("--peak-seconds", type=float, default=4.0)
    ap.add_argument("--peak-reps", type=int, default=10)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="kc", choices=["kc", "reference"])
    ap.add_argument("--workload", default="all", choices=["all"] + sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e pass")
    ap.add_argument("--no-graph", action="store_true",
                    help="gemv: launch the step eagerly instead of replaying it as a CUDA graph")
    ap.add_argument("--gemv-weights", choices=["packed", "tiled"], default="tiled",
                    help="gemv: weights in the reference's packed [N, K/2] layout or the library's "
                         "tile-ordered layout (kc_w4a16_tile_weights, converted once at load)")
    ap.add_argument("--gemv-m", type=int, default=1, choices=[1, 4, 16],
                    help="gemv: activation rows (the decode configuration's batch sizes; the "
                         "headline is M = 1)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="gemv: decoder layers per step (default 32; fewer only for profiling)")
    ap.add_argument("--heat-s", type=float, default=1.5,
                    help="seconds of the same workload run right before the timed region "
                         "(the clock sampler covers it and the timed region)")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)

    if args.tc_calibration:
        tc_calibration()
        return 0
    if args.stream_floor:
        print(json.dumps({"stream_floor": stream_floor()}), flush=True)
        return 0
    if args.peak is not None:
        print(json.dumps(measure_peak(args.peak, args.peak_seconds, args.peak_reps)), flush=True)
        return 0
    if args.impl == "reference":
        run_reference(args)
        return 0

    import torch
    import torch.distributed as dist
    from kc_lib import lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", torch.cuda.current_device())
    l = lib()
    stream = torch.cuda.current_stream()
    s_ptr = ctypes.c_void_p(stream.cuda_stream)

    # a failed correctness gate (agreed by every rank) prints its error line and
    # the run goes on to the next workload, so the headline still prints; the
    # exit status stays non-zero
    rc = 0
    names = _selected(args)
    held = []
    if len(names) > 1 and names[-1] == "gemv":
        names = ["gemv"] + names[:-1]
        rc = run_workload("gemv", args, torch, dist, l, dev, stream, s_ptr, world, rank, local, held) or rc
        names = names[1:]
    for name in names:
        rc = run_workload(name, args, torch, dist, l, dev, stream, s_ptr, world, rank, local) or rc
    for line in held:
        print(line, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())

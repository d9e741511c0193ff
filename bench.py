"""Benchmark of the bo-kernel-tuner hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--secondary auto|none|NAME,NAME...]

Prints ONE JSON line (rank 0).  A step is one pass of a workload's hot path
over one batch of synthetic input already resident in HBM; K steps are
captured in CUDA graphs and replayed between a barrier + synchronize on both
sides (an untimed replay runs right before the timed one, so the GPU is busy
and at clock when the start event is recorded), timed with CUDA events on the
launching stream, max over ranks.

The headline workload (``--workload``, default ``rmsnorm``) gives the line's
top-level ``value``; with the default ``--secondary auto`` the same run also
times the 8192^3 GEMM and the 64-expert MoE step and reports each of them under
``secondary`` with its own roofline, end-to-end rate, CPU baseline, clocks and
parity check.

Workloads:
  rmsnorm    x[4096,4096] bf16 per rank (rows of a G*4096-row matrix split
             across G ranks, no collective: weak scaling); GB/s.
  gemm8192   C = A.B bf16 8192^3; B and C split along N across ranks (A
             replicated, no collective: strong scaling); TFLOP/s.
  gemm2048   2048^3 bf16, replicas; TFLOP/s.  (``_fp16`` variants of both.)
  moe_small  8-expert grouped GEMM, 1528 tokens, replicas; TFLOP/s.
  moe_large  64 experts x [4096, 14336], 16384 tokens top-2 Zipf(1.1):
             one GPU: device routing + gather + grouped GEMM; N GPUs: expert
             parallel with NVLink peer-store dispatch and combine; TFLOP/s.
  rmsnorm_gemm  RMSNorm fused into the 4096 -> 14336 projection; TFLOP/s.

Every workload checks its own output after timing (sampled rows against a
torch fp32 computation on the device, TF32 off, with the reference's gate
tolerances) and reports ``parity``; a mismatch makes the run exit non-zero.
Inputs are larger than L2 (126 MB) or rotated through buffer sets that
together exceed it, so every step reads from HBM.  ``--impl reference`` times
the reference's FP32 CPU path (its worker's torch expressions on CPU tensors,
restated in ``oracle/reference_cpu.py``) on the host cores with the same
``config`` dicts.
"""

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "TFLOP/s (GEMM, MoE grouped GEMM) & RMSNorm GB/s vs B200 peak at 1–8 GPUs"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024
EP_COMM = "peer"  # --ep-comm: expert-parallel dispatch/combine over NVLink peer stores or NCCL
MOE_EXPERTS = None  # --experts: moe_large with fewer experts (small profiling case)
PARAM_OVERRIDES = {}  # --params: launch-parameter overrides for the timed workloads
GEMM_SHAPE = (8192, 8192, 8192)  # --shape of the "gemm" workload
# Rotating input sets together span 4x L2, so a set is long evicted when it is reused.
ROTATION_BYTES = 4 * L2_BYTES
SECONDARY_AUTO = ("gemm8192", "moe_large")


# ----------------------------------------------------------------------------- utilities
def load_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            data = json.loads(path.read_text())
            return data, "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(workload):
    """(DRAM bytes per launch, source) of the dominant kernel from the committed ncu summary."""
    path = REPO / "profiles" / "traffic.json"
    if not path.exists():
        return None, None
    try:
        entry = json.loads(path.read_text()).get(workload)
    except ValueError:
        return None, None
    if not entry:
        return None, None
    return entry.get("bytes_per_launch"), entry.get("source")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def window(self, t0, t1):
        """Clock summary of the samples taken in [t0, t1] (widened by 0.15 s each side)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        lines = list(self.lines)
        window = [line for t, line in lines if t0 - 0.15 <= t <= t1 + 0.15] or \
                 [line for _, line in lines[-5:]]
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in window:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }

    def stop(self):
        if self.proc is None:
            return
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()


def graph_time_ms(stream, fn, count, reps=3):
    """Average device time of ``fn`` (one kernel launch) over ``count`` launches
    captured in one CUDA graph, timed with CUDA events on ``stream``; best of
    ``reps`` replays, each preceded by an untimed replay."""
    import torch

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(count):
            fn(i)
    graph.replay()
    torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            graph.replay()  # untimed: the timed replay starts on a busy GPU
        b.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        e.record(stream)
        e.synchronize()
        t = b.elapsed_time(e) / count
        best = t if best is None else min(best, t)
    del graph
    return best


def paired_graph_times(stream, fn_a, fn_b, count=20, reps=9):
    """Median per-step device time of two step functions, each captured as a
    graph of ``count`` steps and replayed alternately (a, b, a, b, ...) so that
    clock and power drift affect both alike; CUDA events on ``stream``."""
    import torch

    graphs = []
    with torch.cuda.stream(stream):
        for fn in (fn_a, fn_b):  # library set-up (cuBLAS handles, workspaces) before capture
            fn(0)
    torch.cuda.synchronize()
    for fn in (fn_a, fn_b):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(count):
                fn(i)
        graphs.append(g)
    with torch.cuda.stream(stream):
        for g in graphs:
            g.replay()
    torch.cuda.synchronize()
    times = ([], [])
    for _ in range(reps):
        for g, out in zip(graphs, times):
            b, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b.record(stream)
            with torch.cuda.stream(stream):
                g.replay()
            e.record(stream)
            e.synchronize()
            out.append(b.elapsed_time(e) / count)
    del graphs
    return statistics.median(times[0]), statistics.median(times[1])


def cpu_threads():
    return os.cpu_count() or 1


def params_for(kernel, **fixed):
    """Default launch parameters of ``kernel`` with bench overrides (--params) applied."""
    from flashattentionanycard_b200.configs.search_spaces import default_params

    p = dict(default_params(kernel), **fixed)
    p.update(PARAM_OVERRIDES.get(kernel, {}))
    return p


# ----------------------------------------------------------------------------- parity
def gate_check(out, ref, dtype):
    """The reference's FP32 gate (tuner/worker.py:108-116 of the reference:
    finite outputs, |out - ref| <= atol + rtol |ref| with (rtol, atol) = (0.01,
    0.02) for fp16 and (0.02, 0.15) for bf16) plus a normwise relative error
    ||out - ref|| / ||ref|| <= 1e-2."""
    import torch

    rtol, atol = (0.01, 0.02) if dtype == "fp16" else (0.02, 0.15)
    o, r = out.float(), ref.float()
    finite = bool(torch.isfinite(o).all()) and bool(torch.isfinite(r).all())
    diff = (o - r).abs()
    within = bool((diff <= atol + rtol * r.abs()).all())
    norm_r = float(torch.linalg.vector_norm(r))
    normwise = float(torch.linalg.vector_norm(o - r)) / max(norm_r, 1e-30)
    return {"ok": finite and within and normwise <= 1e-2,
            "max_abs_error": float(diff.max()) if diff.numel() else 0.0,
            "normwise_rel_error": normwise, "rtol": rtol, "atol": atol}


def fp32_reference_mode():
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False


def sample_rows(n, count, seed=0):
    """``count`` distinct row indices of [0, n): both ends plus seeded picks."""
    import random

    if n <= count:
        return list(range(n))
    rng = random.Random(seed)
    picks = {0, n - 1, n // 2}
    while len(picks) < count:
        picks.add(rng.randrange(n))
    return sorted(picks)


# ----------------------------------------------------------------------------- configs
# One function per workload, computed on the CPU from the workload's sizes, so
# the GPU arm and the --impl reference arm print the same ``config`` dict.
def rmsnorm_config(world):
    from flashattentionanycard_b200 import workloads

    cfg = workloads.RMSNORM
    m, n = cfg["m"], cfg["n"]
    sets = max(2, math.ceil(ROTATION_BYTES / (2 * m * n * 2)))
    return {"workload": f"rmsnorm_bf16_{m}x{n}_eps1e-6", "rows_per_gpu": m, "hidden": n,
            "total_rows": m * world, "partition": "row-split, no collective",
            "l2": f"rotating {sets} buffer sets ({sets * 2 * m * n * 2 / 2**20:.0f} MiB > L2)",
            "params": params_for("rmsnorm")}


def rotating_sets(per_set_bytes):
    """Input sets to rotate through so that together they exceed L2 by 4x,
    at most 64 (tiny problems stay L2-resident anyway; the cap keeps set-up
    short)."""
    if per_set_bytes >= ROTATION_BYTES:
        return 1
    return min(64, max(1, math.ceil(ROTATION_BYTES / per_set_bytes)))


def gemm_sets(size, n_local):
    return rotating_sets((size * size + 2 * size * n_local) * 2)


def gemm_config(size, dtype, split, world):
    n_local = size // world if split else size
    sets = gemm_sets(size, n_local)
    return {"workload": f"gemm_{dtype}_{size}^3", "m": size, "k": size, "n": size,
            "n_per_gpu": n_local,
            "partition": "N-split, A replicated, no collective" if split else "replicas",
            "l2": "inputs > L2" if sets == 1 else f"rotating {sets} A/C sets",
            "params": params_for("gemm")}


def moe_small_config(world):
    from flashattentionanycard_b200 import workloads

    counts = workloads.MOE_SMALL_COUNTS
    k, n = workloads.MOE_SMALL["k"], workloads.MOE_SMALL["n"]
    nonempty = sum(1 for c in counts if c)
    per_set = (sum(counts) * k + nonempty * k * n + sum(counts) * n) * 2
    sets = max(2, math.ceil(ROTATION_BYTES / per_set))
    return {"workload": "moe_grouped_gemm_bf16_E8_K1024_N2048_T1528",
            "expert_tokens": list(counts), "partition": "replicas",
            "l2": f"rotating {sets} X/W/Y sets", "params": moe_small_params()}


def moe_small_params():
    # Tuned for this single-wave problem (120 tiles of 128 rows on 148 SMs):
    # single-CTA tiles.
    return params_for("moe_grouped_gemm", CTA_GROUP=1, num_stages=4)


def moe_large_cfg():
    from flashattentionanycard_b200 import workloads

    cfg = dict(workloads.MOE_LARGE)
    cfg["experts"] = MOE_EXPERTS or cfg["experts"]
    return cfg


def moe_large_placement(cfg, world):
    import numpy as np

    from flashattentionanycard_b200 import expert_parallel as ep
    from flashattentionanycard_b200 import workloads

    ids = workloads.zipf_routing(cfg["tokens"], cfg["experts"], cfg["topk"], cfg["zipf_s"], 0)
    flat = ids.reshape(-1).numpy()
    placement = ep.plan_placement(np.bincount(flat, minlength=cfg["experts"]), world)
    return ids, placement


def moe_large_gates(cfg):
    """Gate weights of the top-k experts per token: seeded, positive, each
    token's weights summing to 1 (fp32 [tokens, topk])."""
    import torch

    g = torch.Generator().manual_seed(2)
    raw = torch.rand(cfg["tokens"], cfg["topk"], generator=g) + 0.25
    return (raw / raw.sum(1, keepdim=True)).contiguous()


def moe_large_config(world):
    c = moe_large_cfg()
    out = {"workload": f"moe_bf16_E{c['experts']}_K{c['k']}_N{c['n']}_T{c['tokens']}_top2_zipf1.1",
           "partition": "single GPU (all experts local)",
           "step": "route + gather + grouped GEMM + gate-weighted combine (MoE layer; FLOPs "
                   "counted: the grouped GEMM)", "l2": "W 7.5 GB > L2",
           "params": params_for("moe_grouped_gemm")}
    if world > 1:
        _, p = moe_large_placement(c, world)
        step = ("ids put to every rank + device barrier + route + NVLink peer-store dispatch "
                "+ device barrier + grouped GEMM with peer-store epilogue (rows to their token "
                "owners) + device barrier with the gate-weighted combine fused in; no host "
                "collective, steps captured in CUDA graphs"
                if EP_COMM == "peer" else
                "all-gather ids + route + dispatch all-to-all + grouped GEMM + "
                "return all-to-all (NCCL) + gate-weighted combine, eager")
        out.update({
            "partition": f"expert-parallel over {world} GPUs: {p.virtual_experts} virtual "
                         f"experts (hot experts replicated, rows split), LPT placement",
            "step": step, "ep_comm": EP_COMM,
            "rows_per_rank": [int(v) for v in p.rank_rows],
            "max_replicas": int(p.replicas.max()),
        })
    return out


def rmsnorm_gemm_config(world):
    from flashattentionanycard_b200 import workloads

    cfg = workloads.RMSNORM_GEMM
    m, k, n = cfg["m"], cfg["k"], cfg["n"]
    n_local = n // world
    per_set = (m * k + k * n_local + m * n_local) * 2
    sets = max(1, math.ceil(ROTATION_BYTES / per_set)) if per_set < ROTATION_BYTES else 1
    return {"workload": f"rmsnorm_gemm_bf16_{m}x{k}_to_{n}", "m": m, "k": k, "n": n,
            "n_per_gpu": n_local, "eps": cfg["eps"],
            "partition": "N-split, x replicated, no collective",
            "l2": "inputs > L2" if sets == 1 else f"rotating {sets} x/C sets",
            "params": params_for("gemm")}


def gemm_shape_config(world):
    m, n, k = GEMM_SHAPE
    sets = rotating_sets((m * k + k * n + m * n) * 2)
    return {"workload": f"gemm_bf16_{m}x{n}x{k}", "m": m, "n": n, "k": k, "partition": "replicas",
            "l2": "inputs > L2" if sets == 1 else f"rotating {sets} A/C sets",
            "params": params_for("gemm")}


CONFIGS = {
    "rmsnorm": rmsnorm_config,
    "gemm8192": lambda w: gemm_config(8192, "bf16", True, w),
    "gemm2048": lambda w: gemm_config(2048, "bf16", False, w),
    "gemm8192_fp16": lambda w: gemm_config(8192, "fp16", True, w),
    "gemm2048_fp16": lambda w: gemm_config(2048, "fp16", False, w),
    "moe_small": moe_small_config,
    "moe_large": moe_large_config,
    "rmsnorm_gemm": rmsnorm_gemm_config,
    "gemm": lambda w: gemm_shape_config(w),
}
SCALING = {"gemm": "weak", "rmsnorm": "weak", "gemm2048": "weak", "gemm2048_fp16": "weak", "moe_small": "weak",
           "gemm8192": "strong", "gemm8192_fp16": "strong", "moe_large": "strong",
           "rmsnorm_gemm": "strong"}


# ----------------------------------------------------------------------------- workloads
class Rmsnorm:
    name = "rmsnorm"
    unit = "GB/s"
    dtype = "bf16"
    kernel = "rmsnorm_vec_kernel<bf16,4>"
    bound = "hbm"
    launches_per_step = 1

    def __init__(self, device, rank, world):
        import torch

        from flashattentionanycard_b200 import workloads

        cfg = workloads.RMSNORM
        self.m, self.n, self.eps = cfg["m"], cfg["n"], cfg["eps"]
        self.params = params_for("rmsnorm")
        self.bytes_per_step = 2 * self.m * self.n * 2 + self.n * 2  # x in + y out + w
        # Rank r owns rows [r*m, (r+1)*m) of a (world*m)-row matrix: distinct seed per shard.
        x, w = workloads.rmsnorm_inputs(self.m, self.n, "bf16", seed=rank, device=device)
        self.sets = max(2, math.ceil(ROTATION_BYTES / (2 * x.numel() * 2)))
        self.x = [x] + [x.roll(i, 0).contiguous() for i in range(1, self.sets)]
        self.y = [torch.empty_like(x) for _ in range(self.sets)]
        self.w = w

    def step(self, i):
        from flashattentionanycard_b200.kernels import rmsnorm

        s = i % self.sets
        rmsnorm.launch(self.x[s], self.w, self.y[s], self.params, self.eps)

    def value(self, seconds_per_step, world):
        return self.bytes_per_step * world / seconds_per_step / 1e9

    def parity(self):
        import torch

        s = 1 % self.sets
        rows = sample_rows(self.m, 16)
        x = self.x[s][rows].float()
        ref = x * torch.rsqrt(x.square().mean(-1, keepdim=True) + self.eps) * self.w.float()
        out = gate_check(self.y[s][rows], ref, "bf16")
        out["checked"] = f"{len(rows)} sampled rows x {self.n} columns"
        return out

    # e2e through the public API with host buffers
    def e2e_setup(self):
        import torch

        self.h_in = [self.x[0].cpu().pin_memory(), self.w.cpu().pin_memory()]
        self.d_in = [[torch.empty_like(self.x[0]), torch.empty_like(self.w)] for _ in range(2)]
        self.d_out = [torch.empty_like(self.x[0]) for _ in range(2)]
        self.h_out = [torch.empty_like(self.h_in[0]).pin_memory() for _ in range(2)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h_in)
        self.d2h = self.h_out[0].numel() * 2

    def e2e_compute(self, b):
        from flashattentionanycard_b200.kernels import rmsnorm

        x, w = self.d_in[b]
        rmsnorm.launch(x, w, self.d_out[b], self.params, self.eps)


class Gemm:
    unit = "TFLOP/s"
    bound = "tensor"
    launches_per_step = 1

    def __init__(self, device, rank, world, size, dtype="bf16", split=True):
        import torch

        from flashattentionanycard_b200 import workloads

        self.name = f"gemm{size}" + ("_fp16" if dtype == "fp16" else "")
        self.dtype = dtype
        self.size = size
        self.params = params_for("gemm")
        self.kernel = (f"gemm_tc2_kernel<{self.params['BLOCK_N']}>"
                       if self.params.get("CTA_GROUP") == 2
                       else f"gemm_tc_kernel<{self.params['BLOCK_N']},dense>")
        n_local = size // world if split else size
        if split and size % world:
            raise SystemExit("N must divide evenly across ranks")
        a, b = workloads.gemm_inputs(size, size, size, dtype, seed=0, device=device)
        if split:
            b = b[:, rank * n_local:(rank + 1) * n_local].contiguous()
        self.a, self.b = a, b
        self.n_local = n_local
        self.flops_per_step = 2.0 * size * size * n_local
        self.sets = gemm_sets(size, n_local)
        self.A = [a] + [a.roll(i, 0).contiguous() for i in range(1, self.sets)]
        self.C = [torch.empty(size, n_local, device=device, dtype=a.dtype) for _ in range(self.sets)]
        self.split = split

    def step(self, i):
        from flashattentionanycard_b200.kernels import gemm

        s = i % self.sets
        gemm.launch(self.A[s], self.b, self.C[s], self.params)

    def torch_step(self, i):
        import torch

        s = i % self.sets
        torch.mm(self.A[s], self.b, out=self.C[s])

    def value(self, seconds_per_step, world):
        return self.flops_per_step * world / seconds_per_step / 1e12

    def parity(self):
        s = 1 % self.sets
        rows = sample_rows(self.size, 16)
        ref = self.A[s][rows].float() @ self.b.float()
        out = gate_check(self.C[s][rows], ref, self.dtype)
        out["checked"] = f"{len(rows)} sampled rows x {self.n_local} columns of this rank's C"
        return out

    def e2e_setup(self):
        import torch

        self.h_in = [self.a.cpu().pin_memory(), self.b.cpu().pin_memory()]
        self.d_in = [[torch.empty_like(self.a), torch.empty_like(self.b)] for _ in range(2)]
        self.d_out = [torch.empty(self.size, self.n_local, device=self.a.device, dtype=self.a.dtype)
                      for _ in range(2)]
        self.h_out = [torch.empty(self.size, self.n_local, dtype=self.a.dtype).pin_memory()
                      for _ in range(2)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h_in)
        self.d2h = self.h_out[0].numel() * 2

    def e2e_compute(self, b):
        from flashattentionanycard_b200.kernels import gemm

        a, bb = self.d_in[b]
        gemm.launch(a, bb, self.d_out[b], self.params)


class GemmShape(Gemm):
    """C = A.B bf16 of any --shape MxNxK (replicas): e.g. the tall-K shapes
    where split-K pays.  A, B ~ N(0, 1) K^-0.5 as the square configurations."""

    def __init__(self, device, rank, world):
        import torch

        from flashattentionanycard_b200 import workloads

        m, n, k = GEMM_SHAPE
        self.name, self.dtype, self.split = "gemm", "bf16", False
        self.m, self.n_local, self.k = m, n, k
        self.params = params_for("gemm")
        self.kernel = (f"gemm_tc2_kernel<{self.params['BLOCK_N']}>"
                       if self.params.get("CTA_GROUP") == 2
                       else f"gemm_tc_kernel<{self.params['BLOCK_N']},dense>")
        if min(int(self.params.get("SPLIT_K", 1)), -(-k // 64)) >= 4:
            # The library follows the GEMM with its split-K reduction kernel;
            # the timed "kernel" is the pair.
            self.kernel += " + splitk_reduce_kernel"
            self.extra_launches = 1
        a, b = workloads.gemm_inputs(m, n, k, "bf16", seed=0, device=device)
        self.a, self.b = a, b
        self.flops_per_step = 2.0 * m * n * k
        per_set = (m * k + k * n + m * n) * 2
        self.sets = rotating_sets(per_set)
        self.A = [a] + [a.roll(i, 0).contiguous() for i in range(1, self.sets)]
        self.C = [torch.empty(m, n, device=device, dtype=a.dtype) for _ in range(self.sets)]
        self.size = k

    def parity(self):
        s = 1 % self.sets
        rows = sample_rows(self.m, 16)
        out = gate_check(self.C[s][rows], self.A[s][rows].float() @ self.b.float(), "bf16")
        out["checked"] = f"{len(rows)} sampled rows x {self.n_local} columns"
        return out

    def e2e_setup(self):
        import torch

        self.h_in = [self.a.cpu().pin_memory(), self.b.cpu().pin_memory()]
        self.d_in = [[torch.empty_like(self.a), torch.empty_like(self.b)] for _ in range(2)]
        self.d_out = [torch.empty_like(self.C[0]) for _ in range(2)]
        self.h_out = [torch.empty(self.C[0].shape, dtype=self.a.dtype).pin_memory()
                      for _ in range(2)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h_in)
        self.d2h = self.h_out[0].numel() * 2

    def torch_step(self, i):
        import torch

        s = i % self.sets
        torch.mm(self.A[s], self.b, out=self.C[s])


class RmsnormGemm:
    """RMSNorm of x [4096, 4096] fused into the 4096 -> 14336 projection that
    follows it (row-scale pass + row-scaled tcgen05 GEMM with the norm weight
    folded into B); N split across ranks with x replicated (no collective)."""

    name = "rmsnorm_gemm"
    unit = "TFLOP/s"
    bound = "tensor"
    dtype = "bf16"
    launches_per_step = 2  # row-scale pass, row-scaled GEMM

    def __init__(self, device, rank, world):
        import torch

        from flashattentionanycard_b200 import workloads
        from flashattentionanycard_b200.kernels import rmsnorm_gemm

        cfg = workloads.RMSNORM_GEMM
        self.m, self.k, self.n, self.eps = cfg["m"], cfg["k"], cfg["n"], cfg["eps"]
        if self.n % world:
            raise SystemExit("N must divide evenly across ranks")
        self.n_local = self.n // world
        # GROUP_M 16 = all 16 pair row blocks of M = 4096: each weight column block
        # is read from HBM once (DRAM 294 vs 390 MB per launch, 1.6% faster).
        self.params = params_for("gemm", GROUP_M=16)
        self.norm_params = params_for("rmsnorm")
        self.kernel = ("gemm_tc2_kernel<256,rowscale>" if self.params.get("CTA_GROUP") == 2
                       else "gemm_tc_kernel<256,rowscale>")
        x, w, b = workloads.rmsnorm_gemm_inputs(self.m, self.k, self.n, "bf16", seed=0,
                                                device=device)
        self.x, self.w = x, w
        self.b = b[:, rank * self.n_local:(rank + 1) * self.n_local].contiguous()
        # Weight preparation, once per (norm weight, B) pair: not part of a step.
        self.b_folded = rmsnorm_gemm.fold_weight(w, self.b)
        self.flops_per_step = 2.0 * self.m * self.k * self.n_local
        per_set = (x.numel() + self.b.numel() + self.m * self.n_local) * 2
        self.sets = max(1, math.ceil(ROTATION_BYTES / per_set)) if per_set < ROTATION_BYTES else 1
        self.X = [x] + [x.roll(i, 0).contiguous() for i in range(1, self.sets)]
        self.C = [torch.empty(self.m, self.n_local, device=device, dtype=x.dtype)
                  for _ in range(self.sets)]
        self.xn = torch.empty_like(x)
        self.scales = torch.empty(self.m, device=device, dtype=torch.float32)

    def step(self, i):
        from flashattentionanycard_b200.kernels import rmsnorm_gemm

        s = i % self.sets
        rmsnorm_gemm.launch(self.X[s], self.b_folded, self.C[s], self.params, self.eps,
                            scale_workspace=self.scales)

    def dominant_kernel(self, i):
        """The row-scaled GEMM alone (row factors from the last step's pass)."""
        from flashattentionanycard_b200.kernels import rmsnorm_gemm

        s = i % self.sets
        rmsnorm_gemm.gemm_row_scaled(self.X[s], self.b_folded, self.C[s], self.scales,
                                     self.params)

    def unfused_step(self, i):
        """The two-call chain the fused kernel replaces: rmsnorm, then GEMM."""
        from flashattentionanycard_b200.kernels import gemm, rmsnorm

        s = i % self.sets
        rmsnorm.launch(self.X[s], self.w, self.xn, self.norm_params, self.eps)
        gemm.launch(self.xn, self.b, self.C[s], self.params)

    def value(self, seconds_per_step, world):
        return self.flops_per_step * world / seconds_per_step / 1e12

    def parity(self):
        import torch

        s = 0
        self.step(s)  # C[0] from the fused path (the unfused comparison rewrote it)
        torch.cuda.synchronize()
        rows = sample_rows(self.m, 16)
        x = self.X[s][rows].float()
        xn = x * torch.rsqrt(x.square().mean(-1, keepdim=True) + self.eps) * self.w.float()
        out = gate_check(self.C[s][rows], xn @ self.b.float(), "bf16")
        out["checked"] = f"{len(rows)} sampled rows x {self.n_local} columns vs the fp32 chain"
        return out

    def e2e_setup(self):
        import torch

        # Per call the activations travel; the folded weight stays resident,
        # as a layer's weights do.
        self.h_in = [self.x.cpu().pin_memory()]
        self.d_in = [[torch.empty_like(t, device=self.x.device) for t in self.h_in]
                     for _ in range(2)]
        self.d_out = [torch.empty(self.m, self.n_local, device=self.x.device, dtype=self.x.dtype)
                      for _ in range(2)]
        self.h_out = [torch.empty(self.m, self.n_local, dtype=self.x.dtype).pin_memory()
                      for _ in range(2)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h_in)
        self.d2h = self.h_out[0].numel() * 2

    def e2e_compute(self, b):
        from flashattentionanycard_b200.kernels import rmsnorm_gemm

        (x,) = self.d_in[b]
        rmsnorm_gemm.launch(x, self.b_folded, self.d_out[b], self.params, self.eps)


def grouped_kernel_label(params):
    """(kernel, launches) of one grouped GEMM call with ``params``."""
    bn = params.get("BLOCK_N", 256)
    if params.get("CTA_GROUP", 1) == 2:
        return f"gemm_tc2_kernel<{bn},grouped>", 1
    return f"gemm_tc_kernel<{bn},grouped>", 1


def grouped_parity(x, w, offsets, y, rows, dtype="bf16", cols=None):
    """Gate of sampled packed rows of a grouped GEMM output y (expert of a row
    from ``offsets``) against x[row] @ w[expert] in fp32 on the device."""
    import bisect

    import torch

    offs = [int(v) for v in offsets.cpu().tolist()]
    outs, refs = [], []
    for r in rows:
        e = bisect.bisect_right(offs, r) - 1
        wm = w[e] if cols is None else w[e][:, cols]
        refs.append(x[r:r + 1].float() @ wm.float())
        outs.append(y[r:r + 1] if cols is None else y[r:r + 1, cols])
    return gate_check(torch.cat(outs), torch.cat(refs), dtype)


class MoeSmall:
    name = "moe_small"
    unit = "TFLOP/s"
    bound = "hbm"
    dtype = "bf16"

    def __init__(self, device, rank, world):
        import torch

        from flashattentionanycard_b200 import workloads

        counts = workloads.MOE_SMALL_COUNTS
        cfg = workloads.MOE_SMALL
        self.k, self.n = cfg["k"], cfg["n"]
        self.params = moe_small_params()
        self.kernel, self.launches_per_step = grouped_kernel_label(self.params)
        x, w = workloads.moe_inputs(counts, self.k, self.n, "bf16", seed=rank, device=device)
        self.offsets = torch.tensor(workloads.offsets_from_counts(counts), dtype=torch.int32,
                                    device=device)
        t = x.shape[0]
        self.flops_per_step = 2.0 * t * self.k * self.n
        nonempty = sum(1 for c in counts if c)
        self.bytes_per_step = (t * self.k + nonempty * self.k * self.n + t * self.n) * 2
        self.sets = max(2, math.ceil(ROTATION_BYTES / self.bytes_per_step))
        self.X = [x] + [x.roll(i, 0).contiguous() for i in range(1, self.sets)]
        self.W = [w] + [w.roll(i, 1).contiguous() for i in range(1, self.sets)]
        self.Y = [torch.empty(t, self.n, device=device, dtype=x.dtype) for _ in range(self.sets)]
        self.counts = counts
        self.t = t
        self.sm = torch.cuda.get_device_properties(device).multi_processor_count

    def dominant_kernel(self, i):
        """The grouped GEMM call (one launch: single CTAs, or CTA pairs when CTA_GROUP is 2)."""
        self.step(i)

    def step(self, i):
        from flashattentionanycard_b200.kernels import moe_grouped_gemm

        s = i % self.sets
        moe_grouped_gemm.launch(self.X[s], self.W[s], self.offsets, self.Y[s], self.params, self.sm)

    def value(self, seconds_per_step, world):
        return self.flops_per_step * world / seconds_per_step / 1e12

    def parity(self):
        s = 1 % self.sets
        rows = sample_rows(self.t, 24)
        out = grouped_parity(self.X[s], self.W[s], self.offsets, self.Y[s], rows)
        out["checked"] = f"{len(rows)} sampled packed rows x {self.n} columns"
        return out

    def e2e_setup(self):
        import torch

        self.h_in = [self.X[0].cpu().pin_memory(), self.W[0].cpu().pin_memory()]
        self.d_in = [[torch.empty_like(self.X[0]), torch.empty_like(self.W[0])] for _ in range(2)]
        self.d_out = [torch.empty_like(self.Y[0]) for _ in range(2)]
        self.h_out = [torch.empty(self.Y[0].shape, dtype=self.Y[0].dtype).pin_memory()
                      for _ in range(2)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h_in)
        self.d2h = self.h_out[0].numel() * 2

    def e2e_compute(self, b):
        from flashattentionanycard_b200.kernels import moe_grouped_gemm

        x, w = self.d_in[b]
        moe_grouped_gemm.launch(x, w, self.offsets, self.d_out[b], self.params, self.sm)


class MoeLarge:
    name = "moe_large"
    unit = "TFLOP/s"
    bound = "tensor"
    dtype = "bf16"

    def __init__(self, device, rank, world):
        import torch

        from flashattentionanycard_b200 import workloads
        from flashattentionanycard_b200.kernels.moe_routing import MoeRouter

        cfg = moe_large_cfg()
        self.cfg = cfg
        self.world, self.rank = world, rank
        self.params = params_for("moe_grouped_gemm")
        self.kernel, gemm_launches = grouped_kernel_label(self.params)
        # route: count, scan, scatter; gather; GEMM; combine
        self.launches_per_step = 5 + gemm_launches
        self.x, self.w, ids = workloads.moe_large_inputs("bf16", seed=0, device=device,
                                                         experts=cfg["experts"])
        self.ids_cpu = ids
        self.gates_cpu = moe_large_gates(cfg)
        self.sm = torch.cuda.get_device_properties(device).multi_processor_count
        a = ids.numel()
        self.flops_per_step = 2.0 * a * cfg["k"] * cfg["n"]  # whole job, all ranks
        self.graphable = True
        if world > 1:
            self._init_expert_parallel(ids, device)
            return
        self.ids = ids.reshape(-1).to(device)
        self.gates = self.gates_cpu.to(device)
        self.router = MoeRouter(a, cfg["experts"], device)
        self.packed = torch.empty(a, cfg["k"], device=device, dtype=torch.bfloat16)
        self.y = torch.empty(a, cfg["n"], device=device, dtype=torch.bfloat16)
        self.final = torch.empty(cfg["tokens"], cfg["n"], device=device, dtype=torch.bfloat16)

    def _init_expert_parallel(self, ids, device):
        import numpy as np
        import torch
        import torch.distributed as dist

        from flashattentionanycard_b200 import expert_parallel as ep

        cfg, world, rank = self.cfg, self.world, self.rank
        flat = ids.reshape(-1).numpy()
        tpr = cfg["tokens"] // world
        _, self.placement = moe_large_placement(cfg, world)
        self.plan = ep.plan_splits(flat, self.placement, cfg["topk"], tpr)
        local = self.w[ep.local_weight_slices(self.placement, rank)].contiguous()
        # Columns kept for the parity check after the full weights are dropped.
        self.check_cols = list(range(256)) + list(range(cfg["n"] - 256, cfg["n"]))
        self.w_cols = self.w[:, :, self.check_cols].contiguous()
        del self.w  # each rank keeps only its virtual experts' weights
        self.x_local = self.x[rank * tpr:(rank + 1) * tpr].contiguous()
        del self.x
        self.ids_local = ids.reshape(-1)[rank * tpr * cfg["topk"]:(rank + 1) * tpr * cfg["topk"]]
        self.ids_local = self.ids_local.to(torch.int32).to(device)
        self.gates_local = self.gates_cpu[rank * tpr:(rank + 1) * tpr].contiguous().to(device)
        self.comm = EP_COMM
        if self.comm == "peer":
            self.ep = ep.PeerExpertParallelMoE(local, self.placement, self.plan, rank, world,
                                               cfg["topk"], tpr, group=dist.group.WORLD,
                                               params=self.params, sm_count=self.sm)
            # put, 2 barriers, route x3, plan, rowmap, dispatch, grouped GEMM with the
            # peer-scatter epilogue, barrier with the fused combine
            label, gemm_launches = grouped_kernel_label(self.params)
            self.kernel = label.replace(",grouped", ",grouped,scatter")
            self.launches_per_step = 10 + gemm_launches
        else:
            self.ep = ep.ExpertParallelMoE(local, self.placement, self.plan, rank, world,
                                           cfg["topk"], tpr, group=dist.group.WORLD,
                                           params=self.params, sm_count=self.sm)
            # routing/keys/sorts/checks + 4 gathers + grouped GEMM + combine
            self.launches_per_step = 21 + grouped_kernel_label(self.params)[1]
        torch.cuda.empty_cache()
        # Peer path: device barriers only, so whole steps are captured in CUDA
        # graphs.  NCCL path: host collectives between kernels, timed eagerly.
        self.graphable = self.comm == "peer"
        rows = int(self.placement.rank_rows[rank])
        self.kernel_flops = 2.0 * rows * cfg["k"] * cfg["n"]
        self.expected_counts = np.bincount(flat, minlength=cfg["experts"]).astype(np.int32)
        self.expected_local_rows = np.asarray(self.plan.local_rows[rank], dtype=np.int64)

    def step(self, i):
        if self.world > 1:
            self.ep_step(self.x_local, self.ids_local, self.gates_local)
            return
        self.layer(self.x, self.ids, self.gates, self.final)

    def layer(self, x, ids, gates, final):
        """One GPU: route -> gather -> grouped GEMM -> gate-weighted combine."""
        from flashattentionanycard_b200.kernels import moe_grouped_gemm
        from flashattentionanycard_b200.kernels.moe_routing import combine, gather_rows

        self.router(ids)
        gather_rows(x, self.router.perm, self.packed, divisor=self.cfg["topk"])
        moe_grouped_gemm.launch(self.packed, self.w, self.router.offsets, self.y, self.params,
                                self.sm)
        combine(self.y, gates, final, self.router.inv_perm)

    def ep_step(self, x_local, ids_local, gates_local):
        """N GPUs: the expert-parallel step, returning the token-order layer output."""
        from flashattentionanycard_b200.kernels.moe_routing import combine

        if self.comm == "peer":
            return self.ep.forward(x_local, ids_local, gates_local)
        out = self.ep.forward(x_local, ids_local)
        if not hasattr(self, "final_local"):
            import torch

            self.final_local = torch.empty(out.shape[0] // self.cfg["topk"], out.shape[1],
                                           device=out.device, dtype=out.dtype)
        combine(out, gates_local, self.final_local)
        return self.final_local

    def dominant_kernel(self, i):  # noqa: ARG002 - same inputs every launch
        from flashattentionanycard_b200.kernels import moe_grouped_gemm

        if self.world > 1:
            if self.comm == "peer":
                self.ep.compute_and_combine()
            else:
                self.ep.compute()
            return
        moe_grouped_gemm.launch(self.packed, self.w, self.router.offsets, self.y, self.params,
                                self.sm)

    def value(self, seconds_per_step, world):
        return self.flops_per_step / seconds_per_step / 1e12  # whole job at any world size

    def parity(self):
        """Sampled tokens of the layer output (token order, gate-weighted
        combine of the top-k expert rows) against x[t] @ W[e] in fp32 on the
        device, on the first and last 256 output columns; routing bit-exact."""
        import numpy as np
        import torch

        topk = self.cfg["topk"]
        self.step(0)
        torch.cuda.synchronize()
        flat = self.ids_cpu.reshape(-1).numpy()
        cols = list(range(256)) + list(range(self.cfg["n"] - 256, self.cfg["n"]))
        if self.world == 1:
            exact = bool(np.array_equal(self.router.counts.cpu().numpy(),
                                        np.bincount(flat, minlength=self.cfg["experts"])))
            exact = exact and bool(np.array_equal(self.router.perm.cpu().numpy(),
                                                  np.argsort(flat, kind="stable")))
            final, x_tok, first = self.final, self.x, 0
            what = "expert counts and the permutation bit-exact vs numpy bincount / stable argsort"

            def w_cols(e):
                return self.w[e][:, cols]
        else:
            ep = self.ep
            exact = bool(np.array_equal(ep.route_global.counts.cpu().numpy(),
                                        self.expected_counts))
            if self.comm == "peer":
                lrows = np.diff(ep.loffs.cpu().numpy().astype(np.int64))
                exact = exact and bool(np.array_equal(lrows, self.expected_local_rows))
                final = ep.final
            else:
                final = self.final_local
            x_tok = self.x_local
            first = self.rank * x_tok.shape[0]
            what = ("global expert counts and local rows per virtual expert bit-exact vs the "
                    "host plan")

            def w_cols(e):
                return self.w_cols[e]
        tokens = sample_rows(final.shape[0], 32, seed=self.rank)
        refs = []
        for t in tokens:
            acc = torch.zeros(1, len(cols), device=final.device)
            for j in range(topk):
                e = int(flat[(first + t) * topk + j])
                g = float(self.gates_cpu[first + t, j])
                acc += g * (x_tok[t:t + 1].float() @ w_cols(e).float())
            refs.append(acc)
        res = gate_check(final[tokens][:, cols], torch.cat(refs), "bf16")
        res["ok"] = res["ok"] and exact
        res["routing_exact"] = exact
        res["checked"] = (f"rank {self.rank}: {len(tokens)} sampled tokens of the layer output "
                          f"x {len(cols)} columns (first and last 256); {what}")
        return res

    def e2e_setup(self):
        import torch

        if self.world > 1:
            self.hx = self.x_local.cpu().pin_memory()
            self.hids = self.ids_local.cpu().pin_memory()
            self.hg = self.gates_local.cpu().pin_memory()
            rows = self.x_local.shape[0]
            self.hy = torch.empty(rows, self.cfg["n"], dtype=torch.bfloat16).pin_memory()
            self.dx, self.dids = torch.empty_like(self.x_local), torch.empty_like(self.ids_local)
            self.dg = torch.empty_like(self.gates_local)
            self.h2d = self.hx.numel() * 2 + self.hids.numel() * 4 + self.hg.numel() * 4
            self.d2h = self.hy.numel() * 2
            return
        self.h_in = [self.x.cpu().pin_memory(), self.ids.cpu().pin_memory(),
                     self.gates.cpu().pin_memory()]
        self.d_in = [[torch.empty_like(t, device=self.x.device) for t in self.h_in]
                     for _ in range(2)]
        self.d_out = [self.final, torch.empty_like(self.final)]
        self.h_out = [torch.empty(self.final.shape, dtype=self.final.dtype).pin_memory()
                      for _ in range(2)]
        self.h2d = sum(t.numel() * t.element_size() for t in self.h_in)
        self.d2h = self.h_out[0].numel() * 2

    def e2e_step(self):
        """Expert-parallel step with its host copies (not pipelined)."""
        self.dx.copy_(self.hx, non_blocking=True)
        self.dids.copy_(self.hids, non_blocking=True)
        self.dg.copy_(self.hg, non_blocking=True)
        out = self.ep_step(self.dx, self.dids, self.dg)
        self.hy.copy_(out, non_blocking=True)

    def e2e_compute(self, b):
        x, ids, gates = self.d_in[b]
        # One routing state: the compute stream orders consecutive steps.
        self.layer(x, ids, gates, self.d_out[b])

    def release(self):
        """Unmap the peers' buffers (every rank, after a barrier)."""
        if self.world > 1 and hasattr(self.ep, "close"):
            self.ep.close()


WORKLOADS = {
    "rmsnorm": lambda d, r, w: Rmsnorm(d, r, w),
    "gemm8192": lambda d, r, w: Gemm(d, r, w, 8192, "bf16", split=True),
    "gemm2048": lambda d, r, w: Gemm(d, r, w, 2048, "bf16", split=False),
    "gemm8192_fp16": lambda d, r, w: Gemm(d, r, w, 8192, "fp16", split=True),
    "gemm2048_fp16": lambda d, r, w: Gemm(d, r, w, 2048, "fp16", split=False),
    "moe_small": lambda d, r, w: MoeSmall(d, r, w),
    "moe_large": lambda d, r, w: MoeLarge(d, r, w),
    "rmsnorm_gemm": lambda d, r, w: RmsnormGemm(d, r, w),
    "gemm": lambda d, r, w: GemmShape(d, r, w),
}
DEFAULT_STEPS = {"gemm": 200, "rmsnorm": 4000, "gemm8192": 200, "gemm2048": 2000, "gemm8192_fp16": 200,
                 "gemm2048_fp16": 2000, "moe_small": 4000,
                 "moe_large": 100, "rmsnorm_gemm": 400}


# ----------------------------------------------------------------------------- CPU reference
class CpuLeg:
    """The reference's FP32 CPU path of one workload: its own torch expressions
    (oracle.reference_cpu, reference tuner/worker.py:64, 73-74, 88-90) on CPU
    tensors of the 16-bit inputs, intra-op threads over the host cores, on a
    bounded sample; ``step`` returns the work done (bytes or FLOPs)."""

    def __init__(self, name):
        from flashattentionanycard_b200 import workloads

        self.name = name
        self.unit = "GB/s" if name == "rmsnorm" else "TFLOP/s"
        expr = "the reference's FP32 torch expression"
        if name == "rmsnorm":
            cfg = workloads.RMSNORM
            m, n, eps = cfg["m"], cfg["n"], cfg["eps"]
            self.x, self.w = workloads.rmsnorm_inputs(m, n, "bf16", seed=0)
            self.eps = eps
            self.sample = f"{expr} (worker.py:73-74) on the full 4096x4096 bf16 input"
            self.work = 2 * m * n * 2 + n * 2
        elif name == "gemm":
            m, n, k = GEMM_SHAPE
            rows = min(m, 256)
            self.a, self.b = workloads.gemm_inputs(rows, n, k, "bf16", seed=0)
            self.sample = f"{expr} (worker.py:64) on {rows} rows of A x B (K={k}, N={n})"
            self.work = 2.0 * rows * n * k
        elif name.startswith("gemm"):
            size = 8192 if name.startswith("gemm8192") else 2048
            dtype = "fp16" if name.endswith("_fp16") else "bf16"
            rows = 256 if size > 2048 else size
            a, self.b = workloads.gemm_inputs(size, size, size, dtype, seed=0)
            self.a = a[:rows].contiguous()
            self.sample = f"{expr} (worker.py:64) on {rows} rows of A x B (K={size}, N={size})"
            self.work = 2.0 * rows * size * size
        elif name == "moe_small":
            counts = workloads.MOE_SMALL_COUNTS
            k, n = workloads.MOE_SMALL["k"], workloads.MOE_SMALL["n"]
            self.x, self.w = workloads.moe_inputs(counts, k, n, "bf16", seed=0)
            self.starts = workloads.offsets_from_counts(counts)
            self.sample = f"{expr} (worker.py:88-90) on the full 8-expert problem"
            self.work = 2.0 * sum(counts) * k * n
        elif name == "rmsnorm_gemm":
            cfg = workloads.RMSNORM_GEMM
            rows = 256
            x, self.w, self.b = workloads.rmsnorm_gemm_inputs(cfg["m"], cfg["k"], cfg["n"],
                                                              "bf16", seed=0)
            self.x = x[:rows].contiguous()
            self.eps = cfg["eps"]
            self.sample = (f"{expr}s, RMSNorm (worker.py:73-74) of {rows} rows of x then GEMM "
                           f"(worker.py:64) with B (K={cfg['k']}, N={cfg['n']})")
            self.work = 2.0 * rows * cfg["k"] * cfg["n"]
        elif name == "moe_large":
            import torch

            cfg = workloads.MOE_LARGE
            g = torch.Generator().manual_seed(0)
            self.a = torch.randn(256, cfg["k"], generator=g).bfloat16()
            self.b = (0.02 * torch.randn(cfg["k"], cfg["n"], generator=g)).bfloat16()
            self.sample = (f"{expr} of one expert (worker.py:88-90): 256 tokens x "
                           f"W[{cfg['k']}, {cfg['n']}]")
            self.work = 2.0 * 256 * cfg["k"] * cfg["n"]
        else:
            raise ValueError(name)

    def step(self):
        from oracle import reference_cpu as ref

        if self.name == "rmsnorm":
            ref.rmsnorm(self.x, self.w, self.eps)
        elif self.name.startswith("gemm") or self.name == "moe_large":
            ref.gemm(self.a, self.b)
        elif self.name == "moe_small":
            ref.grouped_gemm(self.x, self.w, self.starts)
        elif self.name == "rmsnorm_gemm":
            ref.rmsnorm_gemm(self.x, self.w, self.b, self.eps)
        return self.work


def cpu_measure(name, seconds, min_reps=3):
    """Time the reference's FP32 CPU path of a workload on the host cores for ~``seconds``."""
    from oracle import reference_cpu

    threads = cpu_threads()
    reference_cpu.configure(threads)
    leg = CpuLeg(name)
    leg.step()  # warm
    reps, work, t0 = 0, 0.0, time.perf_counter()
    while reps < min_reps or time.perf_counter() - t0 < seconds:
        work += leg.step()
        reps += 1
    elapsed = time.perf_counter() - t0
    scale = 1e9 if leg.unit == "GB/s" else 1e12
    return {"value": work / elapsed / scale, "unit": leg.unit, "cores": threads, "kind": "port",
            "sample": f"{leg.sample}; {reps} reps in {elapsed:.1f} s"}


def secondary_names(args):
    if args.secondary == "none":
        return []
    if args.secondary == "auto":
        return list(SECONDARY_AUTO) if args.workload == "rmsnorm" else []
    names = [s for s in args.secondary.split(",") if s]
    for s in names:
        if s not in WORKLOADS:
            raise SystemExit(f"unknown secondary workload {s!r}")
    return [s for s in names if s != args.workload]


def reference_entry(name, args, world):
    """One workload of the --impl reference arm: K bounded CPU steps after W untimed ones."""
    from oracle import reference_cpu

    threads = cpu_threads()
    reference_cpu.configure(threads)
    leg = CpuLeg(name)
    times, work = [], 0.0
    for _ in range(args.warmup):
        leg.step()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        work += leg.step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    scale = 1e9 if leg.unit == "GB/s" else 1e12
    value = work / total / scale
    return {
        "workload": name, "value": value, "unit": leg.unit, "ms_per_step": 1e3 * total / args.steps,
        "steps": args.steps, "higher_is_better": True, "scaling": SCALING[name],
        "dtype": "f32", "config": CONFIGS[name](world),
        "cpu_baseline": {"value": value, "unit": leg.unit, "cores": threads, "kind": "port",
                         "sample": leg.sample},
        "e2e": {"value": value, "unit": leg.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference(args):
    """--impl reference: the reference's FP32 CPU path (its torch expressions) on the host."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    head = reference_entry(args.workload, args, world)
    line = {
        "impl": "reference", "metric": METRIC, "value": head["value"], "unit": head["unit"],
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": head["scaling"], "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded inputs of the benchmark configuration shapes)",
        "config": head["config"], "cpu_baseline": head["cpu_baseline"], "e2e": head["e2e"],
    }
    secondary = [reference_entry(name, args, world) for name in secondary_names(args)]
    if secondary:
        line["secondary"] = secondary
    print(json.dumps(line))
    return 0


# ----------------------------------------------------------------------------- GPU arm
def e2e_pipelined(workload, steps):
    """Average ms per step of upload -> compute -> download with two streams and
    double-buffered device tensors (workload.d_in / d_out / h_in / h_out)."""
    import torch

    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    loaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def run(n, begin=None, end=None):
        if begin is not None:
            begin.record(s_in)
        for i in range(n):
            b = i % 2
            if i >= 2:
                s_in.wait_event(consumed[b])
            with torch.cuda.stream(s_in):
                for h, d in zip(workload.h_in, workload.d_in[b]):
                    d.copy_(h, non_blocking=True)
                loaded[b].record(s_in)
            s_out.wait_event(loaded[b])
            with torch.cuda.stream(s_out):
                workload.e2e_compute(b)
                consumed[b].record(s_out)
                workload.h_out[b].copy_(workload.d_out[b], non_blocking=True)
        if end is not None:
            end.record(s_out)
        torch.cuda.synchronize()

    run(2)  # warm: kernel attributes, first touches
    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(steps, begin, end)
    return begin.elapsed_time(end) / steps


def capture_steps(workload, stream, first, count):
    import torch

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(first, first + count):
            workload.step(i)
    return graph


def max_over_ranks(value, world, device):
    import torch
    import torch.distributed as dist

    if world == 1:
        return value
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks_ok(ok, world, device):
    import torch
    import torch.distributed as dist

    if world == 1:
        return ok
    t = torch.tensor([0 if ok else 1], device=device, dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t.item()) == 0


def measure_workload(name, args, steps, ctx):
    """Time one workload (K steps after W warm-up steps), its dominant kernel,
    its end-to-end rate and its parity; returns the result dict (every rank
    takes the same collective steps)."""
    import torch
    import torch.distributed as dist

    from flashattentionanycard_b200 import _native

    world, rank, device, stream = ctx["world"], ctx["rank"], ctx["device"], ctx["stream"]
    sampler, peaks, peak_kind = ctx["sampler"], ctx["peaks"], ctx["peak_kind"]
    workload = WORKLOADS[name](device, rank, world)
    torch.cuda.synchronize()

    # warm-up (eager, outside capture: first calls set kernel attributes)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            workload.step(i)
    stream.synchronize()
    _native.device_status(reset=True)

    graphable = getattr(workload, "graphable", True)
    graphs = []
    if graphable:
        chunk = max(1, min(steps, 250))
        done = 0
        while done < steps:
            count = min(chunk, steps - done)
            graphs.append(capture_steps(workload, stream, done, count))
            done += count
        graphs[0].replay()  # graph upload
        torch.cuda.synchronize()

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # Untimed step(s) right before the start event: the timed region starts on
    # a busy GPU at clock, as the reference's measure() replays once first.
    with torch.cuda.stream(stream):
        if graphable:
            graphs[0].replay()
        else:
            workload.step(0)
    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    begin.record(stream)
    with torch.cuda.stream(stream):
        if graphable:
            for g in graphs:
                g.replay()
        else:
            for i in range(steps):
                workload.step(i)
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    clocks = sampler.window(t0, t1)
    ms = max_over_ranks(begin.elapsed_time(end), world, device)
    code, detail = _native.device_status(reset=True)
    if code:
        raise SystemExit(f"{name}: kernel reported device status {code} (detail {detail})")
    del graphs
    ms_per_step = ms / steps
    value = workload.value(ms_per_step / 1e3, world)

    # Dominant kernel's average launch duration.  A one-kernel step: the timed
    # region itself (events around K launches).  Otherwise a graph of the
    # dominant kernel alone (eager launches for the expert-parallel kernel),
    # timed the same way.
    if workload.launches_per_step == 1:
        kernel_ms = ms_per_step
        kernel_timing = "timed region / launches"
    else:
        # No collectives inside the dominant kernel, so it is captured even
        # for the (eagerly timed) expert-parallel step.
        kernel_ms = graph_time_ms(stream, workload.dominant_kernel, 20)
        kernel_timing = "graph of 20 launches of the dominant kernel alone, best of 3"
    kernel_ms = max_over_ranks(kernel_ms, world, device)
    if workload.unit == "GB/s" or workload.bound == "hbm":
        achieved = workload.bytes_per_step / (kernel_ms / 1e3) / 1e9
        peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        unit_r = "GB/s"
    else:
        flops = getattr(workload, "kernel_flops", workload.flops_per_step)
        achieved = flops / (kernel_ms / 1e3) / 1e12
        peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        unit_r = "TFLOP/s"
    unfused = None
    if hasattr(workload, "unfused_step"):
        fused_ms, unfused_ms = paired_graph_times(stream, workload.step, workload.unfused_step)
        unfused = {"ms_per_step": unfused_ms, "value": workload.value(unfused_ms / 1e3, world),
                   "unit": workload.unit, "fused_ms_per_step": fused_ms,
                   "fused_speedup": unfused_ms / fused_ms,
                   "what": "the two-call chain replaced: rmsnorm.launch then gemm.launch "
                           "(normalised x written to and read back from HBM)",
                   "timing": "paired: graphs of 20 fused / 20 unfused steps replayed "
                             "alternately 9 times each, medians"}
    torch_mm = None
    if args.compare_torch and hasattr(workload, "torch_step"):
        ours_ms, torch_ms = paired_graph_times(stream, workload.step, workload.torch_step)
        torch_mm = {"ms_per_step": torch_ms, "value": workload.value(torch_ms / 1e3, world),
                    "ours_ms_per_step": ours_ms, "speedup_vs_torch": torch_ms / ours_ms,
                    "timing": "paired: graphs of 20 launches of ours / torch.mm replayed "
                              "alternately 9 times each, medians"}
    traffic, traffic_source = profile_traffic(workload.name)
    roofline = {"kernel": workload.kernel, "bound": "hbm" if unit_r == "GB/s" else "tensor",
                "achieved": achieved, "peak": peak, "unit": unit_r, "frac": achieved / peak,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)" if peak_kind == "measured"
                else "fallback", "kernel_ms": kernel_ms, "kernel_timing": kernel_timing,
                "traffic": traffic, "traffic_source": traffic_source}
    if unit_r == "TFLOP/s":
        # `peak` is the burst cuBLAS figure (conservative).  The timed kernels run
        # back to back under the power cap, the regime of the sustained figure,
        # which is reported beside it.
        sustained = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
        roofline["peak_sustained"] = sustained
        roofline["frac_of_sustained"] = achieved / sustained

    # Parity of this run's output (every rank checks its own part).
    fp32_reference_mode()
    parity = workload.parity()
    parity["reference"] = "torch fp32 on the device (TF32 off), the reference's gate tolerances"
    parity["ok"] = all_ranks_ok(bool(parity["ok"]), world, device)

    # End to end through the public API with pinned host buffers.  Every step
    # uploads its inputs and downloads its result; consecutive steps overlap
    # (upload of step i+1 while step i's result downloads: PCIe is full duplex).
    workload.e2e_setup()
    e2e_steps = max(3, min(20, steps))
    pipelined = hasattr(workload, "e2e_compute") and not (
        getattr(workload, "world", 1) > 1 and hasattr(workload, "ep"))
    if pipelined:
        e2e_ms = e2e_pipelined(workload, e2e_steps)
    else:
        with torch.cuda.stream(stream):
            workload.e2e_step()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        eb, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        eb.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(e2e_steps):
                workload.e2e_step()
        ee.record(stream)
        torch.cuda.synchronize()
        e2e_ms = eb.elapsed_time(ee) / e2e_steps
    e2e_ms = max_over_ranks(e2e_ms, world, device)
    e2e = {"value": workload.value(e2e_ms / 1e3, world), "unit": workload.unit,
           "h2d_bytes_per_step": workload.h2d, "d2h_bytes_per_step": workload.d2h,
           "ms_per_step": e2e_ms, "steps": e2e_steps,
           "api": "flashattentionanycard_b200.kernels launch() with pinned host copies",
           "overlap": ("two streams: upload of step i+1 overlaps the download of step i"
                       if pipelined else "sequential per step")}
    result = {
        "workload": name, "value": value, "unit": workload.unit, "steps": steps,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": SCALING[name],
        "dtype": workload.dtype, "config": CONFIGS[name](world), "roofline": roofline,
        "e2e": e2e, "clocks": clocks, "gpu_launches": steps * (workload.launches_per_step + getattr(workload, "extra_launches", 0)),
        "parity": parity,
    }
    if unfused is not None:
        result["unfused"] = unfused
    if torch_mm is not None:
        result["torch_mm"] = torch_mm
    # Free this workload before the next one (peer mappings first, on every rank).
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if hasattr(workload, "release"):
        workload.release()
    if world > 1:
        dist.barrier()
    del workload
    gc.collect()
    torch.cuda.empty_cache()
    return result


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torch.distributed.run")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from flashattentionanycard_b200 import _native

    _native.load()
    peaks, peak_kind = load_peaks()
    sampler = ClockSampler(local)
    sampler.start()  # started well before the first timed region (nvidia-smi start-up)
    ctx = {"world": world, "rank": rank, "device": device, "stream": torch.cuda.Stream(device),
           "sampler": sampler, "peaks": peaks, "peak_kind": peak_kind}
    names = [args.workload] + secondary_names(args)
    results = []
    try:
        for name in names:
            steps = args.steps if args.steps is not None else DEFAULT_STEPS[name]
            results.append(measure_workload(name, args, steps, ctx))
    finally:
        sampler.stop()

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        for i, res in enumerate(results):
            seconds = args.cpu_seconds if i == 0 else args.cpu_seconds / 2
            res["cpu_baseline"] = cpu_measure(res["workload"], seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    parity_ok = all(r["parity"]["ok"] for r in results)
    if rank != 0:
        return 0 if parity_ok else 1
    head = results[0]
    line = {
        "metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
        "steps": head["steps"], "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None,
        "dtype": head["dtype"],
        "data": "synthetic (seeded inputs of the benchmark configuration shapes)",
        "config": head["config"], "roofline": head["roofline"],
        "cpu_baseline": head.get("cpu_baseline"), "e2e": head["e2e"], "clocks": head["clocks"],
        "gpu_launches": head["gpu_launches"], "parity": head["parity"], "impl": "ours",
    }
    for key in ("unfused", "torch_mm"):
        if key in head:
            line[key] = head[key]
    if len(results) > 1:
        line["secondary"] = results[1:]
    print(json.dumps(line))
    if not parity_ok:
        failed = [r["workload"] for r in results if not r["parity"]["ok"]]
        print(f"parity check failed: {failed}", file=sys.stderr)
        return 1
    return 0


def parse_params(text):
    """--params 'gemm:GROUP_M=16,num_stages=5;moe_grouped_gemm:RASTER=2'."""
    out = {}
    for group in filter(None, (text or "").split(";")):
        kernel, _, body = group.partition(":")
        entries = {}
        for item in filter(None, body.split(",")):
            key, _, value = item.partition("=")
            entries[key.strip()] = int(value)
        out[kernel.strip()] = entries
    return out


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="rmsnorm")
    ap.add_argument("--secondary", default="auto",
                    help="'auto' (with the default rmsnorm headline: gemm8192,moe_large), "
                         "'none', or a comma list of workloads timed in the same run")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=None,
                    help="moe_large with this many experts instead of 64 (a smaller case of the "
                         "same kernel, e.g. for ncu captures)")
    ap.add_argument("--ep-comm", choices=("peer", "nccl"), default="peer",
                    help="moe_large at N>1: NVLink peer stores (fused) or NCCL all-to-all")
    ap.add_argument("--shape", default="8192x8192x8192",
                    help="MxNxK of the 'gemm' workload (bf16, replicas)")
    ap.add_argument("--compare-torch", action="store_true",
                    help="GEMM workloads: also time torch.mm (cuBLAS) paired with ours")
    ap.add_argument("--params", default="",
                    help="launch-parameter overrides, e.g. 'gemm:GROUP_M=16;rmsnorm:num_warps=8'")
    args = ap.parse_args()
    global EP_COMM, MOE_EXPERTS, PARAM_OVERRIDES, GEMM_SHAPE
    GEMM_SHAPE = tuple(int(v) for v in args.shape.lower().split("x"))
    if len(GEMM_SHAPE) != 3 or min(GEMM_SHAPE) <= 0:
        raise SystemExit("--shape must be MxNxK")
    EP_COMM = args.ep_comm
    MOE_EXPERTS = args.experts
    PARAM_OVERRIDES = parse_params(args.params)
    if args.impl == "reference" and args.steps is None:
        args.steps = 20
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

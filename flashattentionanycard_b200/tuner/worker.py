"""Disposable CUDA worker: a timeout/illegal access cannot poison the tuner.

Mirror of the reference's ``bo_kernel_tuner/tuner/worker.py`` with the sm_100a
kernels as the candidate implementation.  Same protocol constants, same
``Measurement`` validation, same FP32 correctness gate (``check_output``,
:108-116: fp16 rtol 0.01 / atol 0.02, bf16 rtol 0.02 / atol 0.15) and the same
CUDA-graph timing (``measure``, :135-162).  Differences:

* inputs come from a seeded CPU generator and are copied to the device, and
  the FP32 reference is computed on the CPU by default, so the reference and
  the GPU see bit-identical inputs (the reference draws on the device);
* the candidate is labelled ``CANDIDATE`` ("cuda_sm100a"); "triton" is
  accepted as an alias so the reference's engine can drive this worker;
* ``check_output`` also reports the normwise relative error
  ||out - ref|| / ||ref||;
* the compiled-kernel fields come from ``cudaFuncGetAttributes``.
"""

import json
import math
import statistics
import sys
import time
from dataclasses import dataclass
from pathlib import Path

from flashattentionanycard_b200.configs.search_spaces import Workload

MEASUREMENT_PROTOCOL = "cuda_graph_v2;side_stream_warmup;hot_reused_buffers"
CANDIDATE = "cuda_sm100a"
BASELINES = {
    "gemm": "torch.mm_out",
    "rmsnorm": "torch.nn.functional.rms_norm",
    "moe_grouped_gemm": "torch.mm_out_per_nonempty_expert",
}
PRECISION_POLICY = {
    "tf32": False,
    "fp16_reduced_precision_reduction": False,
    "bf16_reduced_precision_reduction": False,
    "float32_matmul_precision": "highest",
}
TOLERANCES = {"fp16": (0.01, 0.02), "bf16": (0.02, 0.15)}
NORMWISE_LIMIT = 1e-2


@dataclass(frozen=True)
class Measurement:
    warmup: int = 20
    repeats: int = 30
    batch: int = 32
    validation_seeds: int = 2

    def __post_init__(self):
        counts = (self.warmup, self.repeats, self.batch, self.validation_seeds)
        if any(type(v) is not int for v in counts):
            raise ValueError("Measurement counts must be integers")
        if self.warmup < 1 or self.repeats < 3 or self.batch < 1 or self.validation_seeds < 1:
            raise ValueError("Require warmup >= 1, repeats >= 3, batch/seeds >= 1")


def generate_inputs(workload, seed):
    """Seeded N(0,1) inputs in the workload dtype on the CPU, in the reference's
    draw order (worker.py:58-62,71,82)."""
    import torch

    w = workload
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16}[w.dtype]
    generator = torch.Generator(device="cpu").manual_seed(seed)

    def rand(*shape):
        return torch.randn(shape, dtype=dtype, generator=generator)

    if w.kernel == "gemm":
        return {"a": rand(w.m, w.k), "b": rand(w.k, w.n)}
    if w.kernel == "rmsnorm":
        return {"x": rand(w.m, w.n), "weight": rand(w.n)}
    tokens = w.expert_tokens
    x, weight = rand(sum(tokens), w.k), rand(len(tokens), w.k, w.n)
    starts = [0]
    for count in tokens:
        starts.append(starts[-1] + count)
    return {"x": x, "weight": weight, "starts": starts}


def reference_output(workload, inputs):
    """The reference's FP32 formulas (worker.py:64, 73-74, 88-90)."""
    w = workload
    if w.kernel == "gemm":
        return inputs["a"].float() @ inputs["b"].float()
    if w.kernel == "rmsnorm":
        import torch

        x, weight = inputs["x"], inputs["weight"]
        ref = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + w.epsilon)
        return ref * weight.float()
    import torch

    x, weight, starts = inputs["x"], inputs["weight"], inputs["starts"]
    return torch.cat(
        [x[starts[e] : starts[e + 1]].float() @ weight[e].float() for e in range(len(starts) - 1)]
    )


def prepare(workload, device, seed, sm_count, implementation=CANDIDATE, reference_device="cpu"):
    import torch

    if implementation == "triton":
        implementation = CANDIDATE
    if implementation not in (CANDIDATE, "torch"):
        raise ValueError("Unknown implementation")
    baseline = implementation == "torch"
    if not baseline:
        from flashattentionanycard_b200.kernels import gemm, moe_grouped_gemm, rmsnorm

    w = workload
    host = generate_inputs(w, seed)
    if reference_device == "cpu":
        with torch.no_grad():
            ref = reference_output(w, host)
    dev = {k: (v.to(device) if hasattr(v, "to") else v) for k, v in host.items()}
    if reference_device != "cpu":
        ref = reference_output(w, dev)
    ref = ref.to(device)
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16}[w.dtype]

    if w.kernel == "gemm":
        a, b = dev["a"], dev["b"]
        out = torch.empty((w.m, w.n), device=device, dtype=dtype)
        call = (
            (lambda p: torch.mm(a, b, out=out))
            if baseline
            else (lambda p: gemm.launch(a, b, out, p))
        )
    elif w.kernel == "rmsnorm":
        x, weight = dev["x"], dev["weight"]
        out = None if baseline else torch.empty_like(x)
        call = (
            (lambda p: torch.nn.functional.rms_norm(x, (w.n,), weight, w.epsilon))
            if baseline
            else (lambda p: rmsnorm.launch(x, weight, out, p, w.epsilon))
        )
    else:
        x, weight, starts = dev["x"], dev["weight"], dev["starts"]
        tokens = w.expert_tokens
        offsets = torch.tensor(starts, device=device, dtype=torch.int64)
        out = torch.empty((sum(tokens), w.n), device=device, dtype=dtype)
        if baseline:
            views = [
                (x[starts[e] : starts[e + 1]], weight[e], out[starts[e] : starts[e + 1]])
                for e, count in enumerate(tokens)
                if count
            ]

            def call(p):
                for a, b, y in views:
                    torch.mm(a, b, out=y)
                return out
        else:
            call = lambda p: moe_grouped_gemm.launch(x, weight, offsets, out, p, sm_count)  # noqa: E731
    return call, out, ref


def check_output(out, reference, dtype):
    import torch

    rtol, atol = TOLERANCES[dtype]
    if not torch.isfinite(out).all() or not torch.isfinite(reference).all():
        raise AssertionError("Nonfinite output or reference")
    torch.testing.assert_close(out.float(), reference, rtol=rtol, atol=atol)
    delta = (out.float() - reference).abs()
    ref_norm = reference.double().norm().item()
    rel = (out.double() - reference.double()).norm().item() / ref_norm if ref_norm > 0 else 0.0
    if rel > NORMWISE_LIMIT:
        raise AssertionError(f"Normwise relative error {rel:.3e} exceeds {NORMWISE_LIMIT}")
    return {
        "max_abs_error": delta.max().item() if delta.numel() else 0.0,
        "normwise_rel_error": rel,
        "rtol": rtol,
        "atol": atol,
    }


def sample_statistics(samples):
    """Summaries are derived from retained samples; NaN/inf never pass admission."""
    if len(samples) < 3 or any(
        type(x) not in (int, float) or not math.isfinite(x) or x <= 0 for x in samples
    ):
        raise ValueError("Require at least three finite positive CUDA timing samples")
    median = statistics.median(samples)
    return {
        "latency_ms": median,
        "samples_ms": samples,
        "mad_ms": statistics.median(abs(x - median) for x in samples),
        "min_ms": min(samples),
        "max_ms": max(samples),
    }


def measure(call, config):
    import torch

    # Kernel attribute setup (first call per configuration) happens on a side
    # stream before capture, as PyTorch/cuBLAS initialisation does.
    current = torch.cuda.current_stream()
    stream = torch.cuda.Stream()
    stream.wait_stream(current)
    with torch.cuda.stream(stream):
        for _ in range(config.warmup):
            call()
    current.wait_stream(stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(config.batch):
            call()
    graph.replay()
    torch.cuda.synchronize()
    samples = []
    for _ in range(config.repeats):
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record()
        graph.replay()
        end.record()
        end.synchronize()
        samples.append(begin.elapsed_time(end) / config.batch)
    return sample_statistics(samples)


def evaluate(spec):
    import torch

    from flashattentionanycard_b200 import _native
    from flashattentionanycard_b200.tuner.hardware import Hardware

    torch.cuda.set_device(spec["device"])
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    torch.set_float32_matmul_precision("highest")
    hardware = Hardware.detect(spec["device"])
    w = Workload(**spec["workload"])
    config = Measurement(**spec["measurement"])
    p = spec["params"]
    implementation = spec.get("implementation", CANDIDATE)
    if implementation == "triton":
        implementation = CANDIDATE
    baseline = implementation == "torch"
    device = torch.device("cuda", spec["device"])
    started = time.perf_counter()
    validation = []
    for offset in range(config.validation_seeds):
        call, out, ref = prepare(w, device, w.data_seed + offset, hardware.sm_count, implementation)
        if out is not None:
            out.fill_(float("nan"))  # Detect incomplete stores, including ragged tails.
        compiled = call(p)
        torch.cuda.synchronize()
        if not baseline:
            code, detail = _native.device_status(reset=True)
            if code:
                raise RuntimeError(f"kernel reported device status {code} (detail {detail})")
        validation.append(check_output(compiled if baseline else out, ref, w.dtype))
    call, out, ref = prepare(w, device, w.data_seed, hardware.sm_count, implementation)
    shared = None if baseline else int(getattr(compiled.metadata, "shared", 0))
    if shared is not None and shared > hardware.shared_memory_per_block:
        raise RuntimeError("Compiled shared memory exceeds device limit")
    setup_s = time.perf_counter() - started
    result = measure(lambda: call(p), config)
    result.update(
        {
            "validation": validation,
            "setup_compile_validate_s": setup_s,
            "compiled_shared_bytes": shared,
            "compiled_registers": getattr(compiled, "n_regs", None),
            "compiled_spills": getattr(compiled, "n_spills", None),
            "compiled_path": getattr(compiled, "path", None),
            "implementation": BASELINES[w.kernel] if baseline else CANDIDATE,
            "protocol": MEASUREMENT_PROTOCOL,
            "precision_policy": PRECISION_POLICY,
        }
    )
    return result


def evaluate_confirmation(spec):
    """A frozen candidate and its baseline share input seeds and timing settings."""
    from flashattentionanycard_b200.tuner.hardware import Hardware

    order = spec["order"]
    if sorted(order) != ["candidate", "torch"]:
        raise ValueError("Confirmation requires exactly one candidate and one baseline")
    result = {"order": order, "data_seed": spec["workload"]["data_seed"]}
    for name in order:
        result[name] = evaluate(
            dict(spec, implementation=CANDIDATE if name == "candidate" else "torch")
        )
        result[name]["status"] = "ok"
    result["hardware"] = Hardware.detect(spec["device"]).to_dict()
    return result


def main():
    source, destination = map(Path, sys.argv[1:3])
    try:
        spec = json.loads(source.read_text())
        result = evaluate_confirmation(spec) if spec.get("order") is not None else evaluate(spec)
        result["status"] = "ok"
    except Exception as exc:
        import traceback

        traceback.print_exc()
        result = {"status": "error", "error_type": type(exc).__name__, "error": str(exc)}
    destination.write_text(json.dumps(result, allow_nan=False))


if __name__ == "__main__":
    main()

"""Sequential, budget-matched search with complete attempt accounting.

Mirror of the reference's ``bo_kernel_tuner/tuner/engine.py``:

* ``code_fingerprint`` (:28-35) also hashes the CUDA sources and the C ABI
  header, so a kernel change invalidates old studies and warm starts;
* ``isolated_evaluate`` (:80-126) runs one trial in a fresh
  ``python -m flashattentionanycard_b200.tuner.worker`` process with a
  timeout; crashes, timeouts and worker errors become ``EvaluationFailure``;
* ``run_search`` (:181-319) keeps the reference's accounting: pruned,
  failed and non-finite trials consume the attempt budget, a snapshot is
  written atomically after every trial, an existing output is never
  overwritten, a programming error aborts with status ``interrupted``.

Samplers: with Optuna installed, the reference's grid / random / multivariate
TPE over an sqlite study.  Without it (this image has none), grid and random
run on a built-in driver with the same accounting and outputs; TPE and warm
starts require Optuna.

``warm_start`` turns a finished search into a TPE warm-start queue (the
reference's rank-based transfer, ``tuner/transfer.py:11-54``), and ``main`` is a
small command line over this engine.  The reference's own ``run_benchmark``
CLI, engine and worker drive these kernels unchanged through
``flashattentionanycard_b200.dropin`` when the reference is installed.
"""

import argparse

import csv
import hashlib
import importlib.metadata
import json
import math
import os
import platform
import random
import subprocess
import sys
import tempfile
import time
from dataclasses import asdict
from pathlib import Path

from flashattentionanycard_b200.configs.search_spaces import (
    grid_configs,
    grid_size,
    validate_params,
)
from flashattentionanycard_b200.tuner.hardware import prune_reason, resource_estimate
from flashattentionanycard_b200.tuner.worker import MEASUREMENT_PROTOCOL, PRECISION_POLICY, Measurement

PACKAGE = Path(__file__).resolve().parents[1]
FINGERPRINT_GLOBS = (
    ("kernels", "*.py"),
    ("configs", "*.py"),
    ("tuner", "*.py"),
    ("csrc", "*.cu"),
    ("csrc", "*.cuh"),
    ("csrc", "Makefile"),
    ("../include", "*.h"),
)


class EvaluationFailure(RuntimeError):
    pass


def code_fingerprint():
    digest = hashlib.sha256()
    for sub, pattern in FINGERPRINT_GLOBS:
        base = (PACKAGE / sub).resolve()
        for path in sorted(base.glob(pattern)):
            digest.update(f"{sub}/{path.name}".encode())
            digest.update(path.read_bytes())
    return digest.hexdigest()


def have_optuna():
    try:
        import optuna  # noqa: F401
    except ImportError:
        return False
    return True


def environment():
    versions = {}
    for name in ("torch", "numpy", "optuna", "pandas"):
        try:
            versions[name] = importlib.metadata.version(name)
        except importlib.metadata.PackageNotFoundError:
            versions[name] = None
    try:
        smi = subprocess.run(
            [
                "nvidia-smi",
                "--query-gpu=uuid,driver_version,pstate,clocks.sm,clocks.mem,temperature.gpu,power.limit",
                "--format=csv",
            ],
            capture_output=True,
            text=True,
            timeout=5,
        ).stdout
    except (OSError, subprocess.TimeoutExpired):
        smi = "unavailable"
    return {
        "versions": versions,
        "python": sys.version,
        "platform": platform.platform(),
        "nvidia_smi_snapshot": smi,
        "cuda_visible_devices": os.getenv("CUDA_VISIBLE_DEVICES"),
        "library_environment": {k: v for k, v in os.environ.items() if k.startswith("BOKT_")},
    }


def sampler_for(method, space, seed, startup_trials=10):
    import optuna

    if method == "grid":
        return optuna.samplers.GridSampler(space, seed=seed)
    if method == "random":
        return optuna.samplers.RandomSampler(seed=seed)
    if method == "tpe":
        return optuna.samplers.TPESampler(
            seed=seed, multivariate=True, n_startup_trials=startup_trials, constant_liar=False
        )
    raise ValueError("method must be grid, random, or tpe")


def isolated_evaluate(
    workload, hardware, params, measurement, timeout, log_dir, number, *, order=None
):
    """One trial in a fresh worker process (new CUDA context, fresh library load)."""
    log_dir = Path(log_dir)
    log_dir.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory(prefix="bokt-trial-") as directory:
        root = Path(directory)
        source, destination = root / "input.json", root / "output.json"
        source.write_text(
            json.dumps(
                {
                    "workload": asdict(workload),
                    "device": hardware.device,
                    "params": params,
                    "measurement": asdict(measurement),
                    "order": order,
                }
            )
        )
        env = dict(os.environ)
        env["CUDA_CACHE_PATH"] = str(root / "cuda-cache")
        env["PYTHONPATH"] = os.pathsep.join(
            [str(PACKAGE.parent)] + ([env["PYTHONPATH"]] if env.get("PYTHONPATH") else [])
        )
        with (log_dir / f"trial-{number}.log").open("w") as log:
            try:
                run = subprocess.run(
                    [
                        sys.executable,
                        "-m",
                        "flashattentionanycard_b200.tuner.worker",
                        str(source),
                        str(destination),
                    ],
                    env=env,
                    stdout=log,
                    stderr=subprocess.STDOUT,
                    timeout=timeout,
                )
            except subprocess.TimeoutExpired as exc:
                raise EvaluationFailure(f"worker_timeout_after_{timeout}s") from exc
        if run.returncode or not destination.exists():
            raise EvaluationFailure(f"worker_exit_{run.returncode}; see logs/trial-{number}.log")
        result = json.loads(destination.read_text())
        if result["status"] != "ok":
            raise EvaluationFailure(f"{result['error_type']}: {result['error']}")
        return result


def _atomic_json(path, data):
    temporary = path.with_suffix(".tmp")
    temporary.write_text(json.dumps(data, indent=2, allow_nan=False))
    temporary.replace(path)


def export(trials, output, metadata, status, elapsed):
    """Snapshot: result.json (atomic) and trials.csv, as the reference's export."""
    trials = [t for t in trials if t["state"] != "WAITING"]
    completed = [t for t in trials if t["state"] == "COMPLETE"]
    best = min(completed, key=lambda t: t["value"]) if completed else None
    data = {
        "schema_version": 1,
        "status": status,
        "metadata": metadata,
        "elapsed_s": elapsed,
        "attempts": len(trials),
        "successful_evaluations": len(completed),
        "unique_successful_configs": len(
            {json.dumps(t["params"], sort_keys=True) for t in completed}
        ),
        "best": best,
        "trials": trials,
    }
    _atomic_json(output / "result.json", data)
    with (output / "trials.csv").open("w", newline="") as handle:
        writer = csv.DictWriter(handle, fieldnames=["number", "state", "latency_ms", "params", "attrs"])
        writer.writeheader()
        writer.writerows(
            {
                "number": t["number"],
                "state": t["state"],
                "latency_ms": t["value"],
                "params": json.dumps(t["params"]),
                "attrs": json.dumps(t["attrs"]),
            }
            for t in trials
        )
    return data


class _Pruned(Exception):
    pass


def run_search(
    workload,
    hardware,
    space,
    method,
    seed,
    budget,
    output,
    measurement=None,
    time_budget=None,
    trial_timeout=180,
    startup_trials=10,
    warm_params=(),
    transfer=None,
    heuristic_smem=False,
    evaluator=None,
):
    if budget < 1 or seed < 0 or startup_trials < 1 or trial_timeout <= 0:
        raise ValueError("Invalid budget, seed, startup_trials, or timeout")
    if time_budget is not None and time_budget <= 0:
        raise ValueError("time_budget must be positive")
    if method not in ("grid", "random", "tpe"):
        raise ValueError("method must be grid, random, or tpe")
    if warm_params and method != "tpe":
        raise ValueError("Warm start is supported only for TPE")
    effective_budget = min(budget, grid_size(space))
    if len(warm_params) > effective_budget or any(
        not validate_params(p, space) for p in warm_params
    ):
        raise ValueError("Warm-start queue must fit the budget and search space")
    use_optuna = have_optuna()
    if not use_optuna and method == "tpe":
        raise RuntimeError("TPE needs optuna (pip install optuna); grid and random run without it")
    measurement = measurement or Measurement()
    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    if any(output.iterdir()):
        raise ValueError(f"Output directory must be empty: {output}")
    start = time.perf_counter()
    metadata = {
        "workload": workload.signature(),
        "hardware": hardware.to_dict(),
        "search_space": space,
        "method": method,
        "sampler_backend": "optuna" if use_optuna else "builtin",
        "seed": seed,
        "budget": effective_budget,
        "requested_budget": budget,
        "time_budget_s": time_budget,
        "trial_timeout_s": trial_timeout,
        "startup_trials": startup_trials,
        "heuristic_smem": heuristic_smem,
        "measurement": asdict(measurement),
        "transfer": transfer,
        "protocol": "cold_load_per_candidate;" + MEASUREMENT_PROTOCOL,
        "precision_policy": PRECISION_POLICY,
        "code_fingerprint": code_fingerprint(),
        "environment": environment(),
    }
    seen = set()

    def evaluate(params, number, attrs):
        """Objective body shared by both backends; returns the latency."""
        trial_start = time.perf_counter()
        try:
            key = json.dumps(params, sort_keys=True)
            attrs["duplicate"] = key in seen
            seen.add(key)
            attrs["resource_estimate"] = resource_estimate(workload.kernel, params, workload.n)
            reason = prune_reason(hardware, workload.kernel, params, workload.n, heuristic_smem)
            if reason:
                attrs["prune_reason"] = reason
                raise _Pruned(reason)
            remaining = trial_timeout
            if time_budget is not None:
                remaining = min(remaining, time_budget - (time.perf_counter() - start))
                if remaining <= 0:
                    raise EvaluationFailure("wall_time_budget_exhausted")
            result = (
                evaluator(params)
                if evaluator
                else isolated_evaluate(workload, hardware, params, measurement, remaining,
                                       output / "logs", number)
            )
            value = float(result["latency_ms"])
            if not math.isfinite(value) or value <= 0:
                raise EvaluationFailure("invalid_latency")
            attrs["measurement"] = result
            return value
        except EvaluationFailure as exc:
            attrs["failure"] = str(exc)
            raise
        finally:
            attrs["evaluation_wall_s"] = time.perf_counter() - trial_start
            attrs["elapsed_s"] = time.perf_counter() - start

    if use_optuna:
        return _run_optuna(space, method, seed, startup_trials, warm_params, effective_budget,
                           time_budget, output, metadata, start, evaluate)
    return _run_builtin(space, method, seed, effective_budget, time_budget, output, metadata,
                        start, evaluate)


def _run_builtin(space, method, seed, attempts, time_budget, output, metadata, start, evaluate):
    """Grid (seeded order over unvisited points) or random sampling without optuna."""
    rng = random.Random(seed)
    grid = list(grid_configs(space))
    rng.shuffle(grid)
    trials = []
    status = "interrupted"
    try:
        for number in range(attempts):
            if time_budget is not None and time.perf_counter() - start >= time_budget:
                break
            if method == "grid":
                params = grid[number]
            else:
                params = {name: rng.choice(choices) for name, choices in space.items()}
            trial = {"number": number, "state": "RUNNING", "value": None, "params": params,
                     "attrs": {}}
            trials.append(trial)
            try:
                trial["value"] = evaluate(params, number, trial["attrs"])
                trial["state"] = "COMPLETE"
            except _Pruned:
                trial["state"] = "PRUNED"
            except EvaluationFailure:
                trial["state"] = "FAIL"
            export(trials, output, metadata, "running", time.perf_counter() - start)
        status = "complete" if any(t["state"] == "COMPLETE" for t in trials) else "failed"
    finally:
        for t in trials:
            if t["state"] == "RUNNING":
                t["state"] = "FAIL"
        data = export(trials, output, metadata, status, time.perf_counter() - start)
    return data


def _run_optuna(space, method, seed, startup_trials, warm_params, attempts, time_budget, output,
                metadata, start, evaluate):
    import optuna

    study = optuna.create_study(
        direction="minimize",
        sampler=sampler_for(method, space, seed, startup_trials),
        study_name="kernel",
        storage=f"sqlite:///{(output / 'study.sqlite3').resolve()}",
    )
    study.set_user_attr("metadata", metadata)
    for rank, params in enumerate(warm_params):
        study.enqueue_trial(params, user_attrs={"warm_start_rank": rank})

    def snapshot():
        return [
            {"number": t.number, "state": t.state.name, "value": t.value, "params": t.params,
             "attrs": t.user_attrs}
            for t in study.trials
        ]

    def objective(trial):
        params = {name: trial.suggest_categorical(name, choices) for name, choices in space.items()}
        attrs = {}
        try:
            return evaluate(params, trial.number, attrs)
        except _Pruned as exc:
            raise optuna.TrialPruned(str(exc)) from exc
        finally:
            for key, value in attrs.items():
                trial.set_user_attr(key, value)

    def checkpoint(study, trial):
        export(snapshot(), output, metadata, "running", time.perf_counter() - start)
        if time_budget is not None and time.perf_counter() - start >= time_budget:
            study.stop()

    status = "interrupted"
    try:
        remaining = None if time_budget is None else max(0, time_budget - (time.perf_counter() - start))
        study.optimize(objective, n_trials=attempts, timeout=remaining, n_jobs=1,
                       catch=(EvaluationFailure,), callbacks=[checkpoint])
        status = ("complete" if any(t.state == optuna.trial.TrialState.COMPLETE
                                    for t in study.trials) else "failed")
    finally:
        data = export(snapshot(), output, metadata, status, time.perf_counter() - start)
    return data


# ----------------------------------------------------------------------------- warm start
def _usable(trial):
    value = trial.get("value")
    return (trial.get("state") == "COMPLETE" and isinstance(value, (int, float))
            and math.isfinite(value) and value > 0)


def warm_start(result_path, workload, space, top_k, hardware, prune):
    """TPE warm-start queue from a finished search: the ``top_k`` fastest
    distinct configurations of the source that are legal here.

    Only the source's ranking transfers, never its latencies: the queued
    configurations are measured again on this device.  The source must be a
    complete schema-1 result for the same workload signature, search space and
    code fingerprint (kernels, search space and measurement code unchanged).
    ``prune(params)`` returns a reason (truthy) for configurations illegal on
    the target.  Returns (queue, provenance)."""
    if top_k < 1:
        raise ValueError("top_k must be at least 1")
    raw = Path(result_path).read_bytes()
    source = json.loads(raw)
    if source.get("schema_version") != 1 or source.get("status") != "complete":
        raise ValueError("Warm start needs a complete schema-1 search result")
    meta = source.get("metadata", {})
    if meta.get("workload") != workload.signature() or meta.get("search_space") != space:
        raise ValueError("Warm start source workload or search space mismatch")
    if meta.get("code_fingerprint") != code_fingerprint():
        raise ValueError("Warm start source was measured with different kernel code")
    queue = []
    for trial in sorted(filter(_usable, source.get("trials", [])), key=lambda t: t["value"]):
        params = trial["params"]
        if params in queue or not validate_params(params, space) or prune(params):
            continue
        queue.append(params)
        if len(queue) == top_k:
            break
    if not queue:
        raise ValueError("No legal source configurations available")
    provenance = {
        "source_sha256": hashlib.sha256(raw).hexdigest(),
        "source_hardware": meta.get("hardware"),
        "target_hardware": hardware.to_dict(),
        "requested_top_k": top_k,
        "enqueued": len(queue),
        "strategy": "ranked_parameters_remeasured_on_target",
    }
    return queue, provenance


# ----------------------------------------------------------------------------- command line
def main(argv=None):
    """``python -m flashattentionanycard_b200.tuner.engine --kernel gemm --m 2048 ...``:
    one search over the kernel's launch space, trials in fresh worker processes,
    result.json / trials.csv in ``--output``."""
    from flashattentionanycard_b200.configs.search_spaces import Workload, search_space
    from flashattentionanycard_b200.tuner.hardware import Hardware

    ap = argparse.ArgumentParser(description="Search the sm_100a kernels' launch parameters.")
    ap.add_argument("--kernel", choices=("gemm", "rmsnorm", "moe_grouped_gemm"), default="gemm")
    ap.add_argument("--dtype", choices=("fp16", "bf16"), default="bf16")
    ap.add_argument("--m", type=int, default=1024)
    ap.add_argument("--n", type=int, default=1024)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--expert-tokens", default="64,128,256,512")
    ap.add_argument("--epsilon", type=float, default=1e-6)
    ap.add_argument("--data-seed", type=int, default=17)
    ap.add_argument("--method", choices=("grid", "random", "tpe"), default="grid")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--trials", type=int, default=50)
    ap.add_argument("--profile", choices=("full", "smoke"), default="full")
    ap.add_argument("--output", type=Path, required=True)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--time-budget", type=float, default=None)
    ap.add_argument("--trial-timeout", type=float, default=180)
    ap.add_argument("--warm-start", type=Path, default=None, help="result.json of a finished search")
    ap.add_argument("--top-k", type=int, default=5)
    ap.add_argument("--measurement", default="20,30,32,2",
                    help="warmup,repeats,batch,validation_seeds")
    ap.add_argument("--dry-run", action="store_true", help="print the plan, touch no GPU")
    args = ap.parse_args(argv)
    try:
        workload = Workload(args.kernel, args.m, args.n, args.k, args.dtype,
                            tuple(int(x) for x in args.expert_tokens.split(",")), args.epsilon,
                            args.data_seed)
        space = search_space(args.kernel, args.profile)
        measurement = Measurement(*(int(x) for x in args.measurement.split(",")))
        if args.warm_start is not None and args.method != "tpe":
            raise ValueError("--warm-start seeds a TPE search (--method tpe)")
    except ValueError as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 2
    print(json.dumps({"workload": workload.signature(), "grid_size": grid_size(space),
                      "method": args.method, "attempt_budget": min(args.trials, grid_size(space))}))
    if args.dry_run:
        return 0
    hardware = Hardware.detect(args.device)
    queue, provenance = (), None
    if args.warm_start is not None:
        queue, provenance = warm_start(
            args.warm_start, workload, space, args.top_k, hardware,
            lambda p: prune_reason(hardware, args.kernel, p, args.n))
    result = run_search(workload, hardware, space, args.method, args.seed, args.trials,
                        args.output, measurement, args.time_budget, args.trial_timeout,
                        warm_params=queue, transfer=provenance)
    best = result["best"]
    print(json.dumps({"status": result["status"], "attempts": result["attempts"],
                      "successful": result["successful_evaluations"],
                      "best_ms": best["value"] if best else None,
                      "best_params": best["params"] if best else None}))
    return 0 if result["status"] == "complete" else 1


if __name__ == "__main__":
    sys.exit(main())

"""Paired confirmation of a frozen search winner against the PyTorch baseline.

Same protocol and evidence files as the reference's
``bo_kernel_tuner/tuner/confirmation.py`` (PROTOCOL string :35, FILES :36,
plan :96-107, bootstrap summary :126-147, CSV :150-159, CPU-only verification
:162-197), with the sm_100a kernels as the candidate:

* the source is a completed search (``run_benchmark`` / ``engine.run_search``
  ``result.json``) whose code fingerprint, protocol and precision policy match
  the current tree;
* every repetition is one fresh worker process that measures the frozen
  candidate and the torch baseline back to back on held-out input seeds
  (never a search validation seed), alternating which goes first;
* only complete, validated pairs enter the summary: the median of the paired
  speedups baseline / candidate and a descriptive percentile bootstrap over
  pairs;
* ``verify`` recomputes plan, pair validation, summary, CSV and the sha256
  receipt from the files alone, without CUDA.

``bench.py`` and ``tuner/scaling.py`` apply the same pairing to multi-GPU
scaling (1 vs G GPUs) and to the CPU reference arm.
"""

import argparse
import csv
import hashlib
import io
import json
import math
import random
import statistics
import time
from dataclasses import asdict, replace
from pathlib import Path

from flashattentionanycard_b200.configs.search_spaces import Workload, validate_params
from flashattentionanycard_b200.tuner.engine import (
    _atomic_json,
    code_fingerprint,
    environment,
    isolated_evaluate,
)
from flashattentionanycard_b200.tuner.hardware import Hardware
from flashattentionanycard_b200.tuner.worker import (
    BASELINES,
    CANDIDATE,
    MEASUREMENT_PROTOCOL,
    PRECISION_POLICY,
    TOLERANCES,
    Measurement,
    sample_statistics,
)

PROTOCOL = "paired_confirmation_v1;fresh_process_per_pair;held_out_inputs;balanced_order"
SEARCH_PROTOCOL = "cold_load_per_candidate;" + MEASUREMENT_PROTOCOL
FILES = ("source-result.json", "confirmation.json", "pairs.csv")
BOOTSTRAP_DRAWS = 5000
BOOTSTRAP_SEED = 0
INTERVAL_METHOD = "descriptive_percentile_bootstrap_of_pairs;5000_draws;seed=0"


class ConfirmationError(ValueError):
    pass


# ------------------------------------------------------------------ validation
def check_measurement(result, measurement, dtype, implementation):
    """A worker measurement is admissible only if it is complete and self-consistent."""
    samples = result.get("samples_ms", [])
    try:
        summary = sample_statistics(samples)
    except ValueError as exc:
        raise ConfirmationError(f"bad timing samples: {exc}") from exc
    problems = []
    if result.get("status") != "ok":
        problems.append("status")
    if result.get("implementation") != implementation:
        problems.append("implementation")
    if result.get("protocol") != MEASUREMENT_PROTOCOL:
        problems.append("protocol")
    if result.get("precision_policy") != PRECISION_POLICY:
        problems.append("precision_policy")
    if len(samples) != measurement.repeats:
        problems.append("sample count")
    if any(result.get(key) != value for key, value in summary.items()):
        problems.append("summary")
    validation = result.get("validation", [])
    if len(validation) != measurement.validation_seeds:
        problems.append("validation seeds")
    for entry in validation:
        error = entry.get("max_abs_error")
        if type(error) not in (int, float) or not math.isfinite(error) or error < 0:
            problems.append("max_abs_error")
        if (entry.get("rtol"), entry.get("atol")) != TOLERANCES[dtype]:
            problems.append("tolerance")
    if problems:
        raise ConfirmationError("inconsistent measurement: " + ", ".join(sorted(set(problems))))


def freeze_source(raw, require_current=True):
    """Parse a completed search and return (source, workload, measurement)."""
    source = json.loads(raw)
    if source.get("schema_version") != 1 or source.get("status") != "complete":
        raise ConfirmationError("confirmation needs a completed schema-1 search result")
    meta = source["metadata"]
    workload = Workload(**meta["workload"])
    measurement = Measurement(**meta["measurement"])
    if meta.get("protocol") != SEARCH_PROTOCOL or meta.get("precision_policy") != PRECISION_POLICY:
        raise ConfirmationError("the search used another measurement protocol")
    if require_current and meta.get("code_fingerprint") != code_fingerprint():
        raise ConfirmationError("kernel or tuner code changed since the search; search again")
    trials = source["trials"]
    complete = [t for t in trials if t["state"] == "COMPLETE"]
    finite = all(type(t["value"]) in (int, float) and math.isfinite(t["value"]) and t["value"] > 0
                 for t in complete)
    if (not complete or not finite or source["attempts"] != len(trials)
            or source["successful_evaluations"] != len(complete)):
        raise ConfirmationError("search trial accounting or latencies are invalid")
    best = min(complete, key=lambda t: t["value"])
    if source["best"] != best or not validate_params(best["params"], meta["search_space"]):
        raise ConfirmationError("recorded winner is not the best successful trial")
    check_measurement(best["attrs"]["measurement"], measurement, workload.dtype, CANDIDATE)
    if best["value"] != best["attrs"]["measurement"]["latency_ms"]:
        raise ConfirmationError("winner latency differs from its samples")
    return source, workload, measurement


def make_plan(workload, measurement, repetitions):
    """Held-out seeds (disjoint from the search's and from each other), balanced order."""
    if type(repetitions) is not int or repetitions < 3:
        raise ConfirmationError("need at least three paired repetitions")
    plan = []
    for i in range(repetitions):
        first = "candidate" if i % 2 == 0 else "torch"
        second = "torch" if first == "candidate" else "candidate"
        plan.append({
            "repetition": i,
            "data_seed": workload.data_seed + (i + 1) * measurement.validation_seeds,
            "order": [first, second],
        })
    return plan


def same_hardware(a, b):
    """Identity fields that must match between source and pairs (not the device index)."""
    def strip(h):
        return {k: v for k, v in h.items() if k != "device"}

    return strip(a) == strip(b)


def check_pair(pair, planned, hardware, workload, measurement):
    if pair.get("status") != "ok":
        raise ConfirmationError("pair did not complete")
    if pair.get("order") != planned["order"] or pair.get("data_seed") != planned["data_seed"]:
        raise ConfirmationError("pair order or seed differs from the plan")
    if not same_hardware(pair.get("hardware", {}), hardware):
        raise ConfirmationError("pair ran on another GPU")
    check_measurement(pair["candidate"], measurement, workload.dtype, CANDIDATE)
    check_measurement(pair["torch"], measurement, workload.dtype, BASELINES[workload.kernel])


# ------------------------------------------------------------------ statistics
def bootstrap_interval(ratios, draws=BOOTSTRAP_DRAWS, seed=BOOTSTRAP_SEED):
    """(2.5%, 97.5%) percentiles of the median over resampled pairs (linear
    interpolation between order statistics)."""
    rng = random.Random(seed)
    medians = sorted(statistics.median(rng.choices(ratios, k=len(ratios))) for _ in range(draws))

    def at(q):
        pos = (len(medians) - 1) * q
        lo = math.floor(pos)
        hi = math.ceil(pos)
        return medians[lo] + (medians[hi] - medians[lo]) * (pos - lo)

    return at(0.025), at(0.975)


def summarize(pairs):
    speedups = [p["torch"]["latency_ms"] / p["candidate"]["latency_ms"] for p in pairs]
    low, high = bootstrap_interval(speedups)
    return {
        "paired_repetitions": len(pairs),
        "candidate_median_ms": statistics.median(p["candidate"]["latency_ms"] for p in pairs),
        "baseline_median_ms": statistics.median(p["torch"]["latency_ms"] for p in pairs),
        "median_paired_speedup": statistics.median(speedups),
        "paired_speedups": speedups,
        "ci95_low": low,
        "ci95_high": high,
        "interval_method": INTERVAL_METHOD,
        "scope": "One frozen configuration on one device/session, not search-seed or fleet variance",
    }


def pairs_csv(pairs):
    buffer = io.StringIO(newline="")
    out = csv.writer(buffer, lineterminator="\n")
    out.writerow(["repetition", "data_seed", "first", "candidate_ms", "baseline_ms", "speedup"])
    for i, pair in enumerate(pairs):
        c, b = pair["candidate"]["latency_ms"], pair["torch"]["latency_ms"]
        out.writerow([i, pair["data_seed"], pair["order"][0], c, b, b / c])
    return buffer.getvalue()


def receipt(output, files=FILES):
    return {name: hashlib.sha256((Path(output) / name).read_bytes()).hexdigest() for name in files}


# ------------------------------------------------------------------ verification
def verify_confirmation(output):
    """Recompute everything from the evidence files (no CUDA); return the summary."""
    output = Path(output)
    raw = (output / "source-result.json").read_bytes()
    source, workload, measurement = freeze_source(raw, require_current=False)
    report = json.loads((output / "confirmation.json").read_text())
    plan = make_plan(workload, measurement, report["repetitions"])
    expected = {
        "schema_version": 1,
        "status": "complete",
        "protocol": PROTOCOL,
        "source_sha256": hashlib.sha256(raw).hexdigest(),
        "selected_params": source["best"]["params"],
        "search_best_ms": source["best"]["value"],
        "baseline": BASELINES[workload.kernel],
        "plan": plan,
        "measurement": asdict(measurement),
        "code_fingerprint": source["metadata"]["code_fingerprint"],
        "precision_policy": PRECISION_POLICY,
    }
    mismatched = [k for k, v in expected.items() if report.get(k) != v]
    if (mismatched or not same_hardware(report["hardware"], source["metadata"]["hardware"])
            or report["hardware"].get("uuid", "unknown") == "unknown"
            or report["environment"]["versions"] != source["metadata"]["environment"]["versions"]
            or len(report["pairs"]) != len(plan)):
        raise ConfirmationError("confirmation provenance or completeness mismatch "
                                f"({', '.join(mismatched) or 'hardware/environment/pairs'})")
    for pair, planned in zip(report["pairs"], plan):
        check_pair(pair, planned, report["hardware"], workload, measurement)
    if report.get("summary") != summarize(report["pairs"]):
        raise ConfirmationError("summary differs from the paired evidence")
    if (output / "pairs.csv").read_text() != pairs_csv(report["pairs"]):
        raise ConfirmationError("pairs.csv differs from the paired evidence")
    if json.loads((output / "receipt.json").read_text()) != receipt(output):
        raise ConfirmationError("receipt mismatch")
    return report["summary"]


# ------------------------------------------------------------------ driver
def confirm(source_path, output, device=0, repetitions=6, timeout=180, dry_run=False,
            evaluate_pair=None):
    """Run the paired plan.  ``evaluate_pair(workload, hardware, params, measurement,
    timeout, log_dir, number, order=...)`` defaults to a fresh worker process."""
    raw = Path(source_path).read_bytes()
    source, workload, measurement = freeze_source(raw)
    plan = make_plan(workload, measurement, repetitions)
    if type(device) is not int or device < 0 or not math.isfinite(timeout) or timeout <= 0:
        raise ConfirmationError("invalid device or worker timeout")
    output = Path(output)
    if output.exists():
        raise ConfirmationError("use a new confirmation output directory")
    if dry_run:
        return {"baseline": BASELINES[workload.kernel], "plan": plan,
                "worker_timeout_sum_s": repetitions * timeout}
    hardware = Hardware.detect(device)
    env = environment()
    if (hardware.uuid == "unknown"
            or not same_hardware(hardware.to_dict(), source["metadata"]["hardware"])
            or env["versions"] != source["metadata"]["environment"]["versions"]):
        raise ConfirmationError("confirmation needs the search's GPU and software versions")
    evaluate_pair = evaluate_pair or isolated_evaluate
    output.mkdir(parents=True)
    (output / "source-result.json").write_bytes(raw)
    report = {
        "schema_version": 1,
        "status": "running",
        "protocol": PROTOCOL,
        "code_fingerprint": code_fingerprint(),
        "source_sha256": hashlib.sha256(raw).hexdigest(),
        "selected_params": source["best"]["params"],
        "search_best_ms": source["best"]["value"],
        "baseline": BASELINES[workload.kernel],
        "hardware": hardware.to_dict(),
        "environment": env,
        "precision_policy": PRECISION_POLICY,
        "measurement": asdict(measurement),
        "repetitions": repetitions,
        "worker_timeout_s": timeout,
        "plan": plan,
        "pairs": [],
        "summary": None,
    }
    started = time.perf_counter()
    try:
        _atomic_json(output / "confirmation.json", report)
        for planned in plan:
            pair = evaluate_pair(replace(workload, data_seed=planned["data_seed"]), hardware,
                                 report["selected_params"], measurement, timeout,
                                 output / "logs", planned["repetition"], order=planned["order"])
            check_pair(pair, planned, hardware.to_dict(), workload, measurement)
            report["pairs"].append(pair)
            _atomic_json(output / "confirmation.json", report)
        report["status"] = "complete"
        report["summary"] = summarize(report["pairs"])
        (output / "pairs.csv").write_text(pairs_csv(report["pairs"]))
    except BaseException as exc:
        report["status"] = "interrupted" if isinstance(exc, KeyboardInterrupt) else "failed"
        report["summary"] = None
        report["error"] = f"{type(exc).__name__}: {exc}"
        raise
    finally:
        report["elapsed_s"] = time.perf_counter() - started
        _atomic_json(output / "confirmation.json", report)
    _atomic_json(output / "receipt.json", receipt(output))
    verify_confirmation(output)
    return report


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("source", nargs="?", type=Path, help="completed search result.json")
    parser.add_argument("--output", type=Path)
    parser.add_argument("--device", type=int, default=0)
    parser.add_argument("--repetitions", type=int, default=6)
    parser.add_argument("--timeout", type=float, default=180)
    parser.add_argument("--dry-run", action="store_true")
    parser.add_argument("--verify", type=Path, help="verify a confirmation directory (no CUDA)")
    args = parser.parse_args(argv)
    try:
        if args.verify:
            if args.source or args.output or args.dry_run:
                raise ConfirmationError("--verify takes no execution inputs")
            result = verify_confirmation(args.verify)
        else:
            if args.source is None or args.output is None:
                raise ConfirmationError("source and --output are required")
            result = confirm(args.source, args.output, args.device, args.repetitions,
                             args.timeout, args.dry_run)
        print(json.dumps(result, indent=2, allow_nan=False))
        return 0
    except (ValueError, RuntimeError, OSError, KeyError, TypeError) as exc:
        print(f"Confirmation failed: {exc}")
        return 1


if __name__ == "__main__":
    raise SystemExit(main())

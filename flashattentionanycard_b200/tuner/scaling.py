"""Paired scaling confirmation: 1 vs G GPUs, and the CPU reference vs the GPU path.

The reference's paired protocol (``bo_kernel_tuner/tuner/confirmation.py``:
fresh process per measurement, balanced order, only complete pairs, median of
paired ratios with a descriptive percentile bootstrap, evidence files with a
sha256 receipt, CPU-only verification) applied to ``bench.py`` runs:

* ``mode="gpus"``: each repetition runs the benchmark once on 1 GPU and once on
  G GPUs (``torch.distributed.run``, one rank per GPU), alternating which runs
  first.  Paired ratio = value(G) / value(1) (``value`` is the whole-job rate of
  the JSON contract), efficiency = ratio / G.
* ``mode="cpu"``: each repetition runs ``--impl reference`` (the reference's CPU
  path on the host cores) and ``--impl ours`` at N = 1.  Paired ratio = our
  end-to-end rate (host buffers in and out, the contract's ``e2e``) / the
  reference's rate.

A run whose JSON line is missing, malformed, reports another configuration or
throttled clocks (hw_slowdown / hw_thermal_slowdown / sw_thermal_slowdown) is a
failed run: the confirmation stops and publishes no ratio.
"""

import argparse
import csv
import hashlib
import io
import json
import math
import os
import socket
import statistics
import subprocess
import sys
import time
from pathlib import Path

from flashattentionanycard_b200.tuner.confirmation import (
    ConfirmationError,
    bootstrap_interval,
    INTERVAL_METHOD,
)
from flashattentionanycard_b200.tuner.engine import _atomic_json, code_fingerprint, environment

PROTOCOL = "paired_scaling_v1;fresh_processes_per_run;balanced_order;bench_json_contract"
FILES = ("scaling.json", "pairs.csv")
REPO = Path(__file__).resolve().parents[2]
REJECTED_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")


def make_plan(mode, gpus, repetitions):
    if mode not in ("gpus", "cpu"):
        raise ConfirmationError("mode must be 'gpus' or 'cpu'")
    if type(repetitions) is not int or repetitions < 3:
        raise ConfirmationError("need at least three paired repetitions")
    if mode == "gpus" and (type(gpus) is not int or gpus < 2):
        raise ConfirmationError("gpus mode compares 1 GPU with G >= 2 GPUs")
    arms = ("one", "many") if mode == "gpus" else ("reference", "ours")
    return [{"repetition": i, "order": list(arms if i % 2 == 0 else arms[::-1])}
            for i in range(repetitions)]


def arm_spec(mode, arm, gpus):
    """(n_gpus, impl) of one arm."""
    if mode == "gpus":
        return (1 if arm == "one" else gpus), "ours"
    return 1, ("reference" if arm == "reference" else "ours")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def bench_command(workload, n, impl, steps, warmup, timeout):
    """The benchmark's own launch line for one arm (steps None: its per-workload default)."""
    args = ["bench.py", "--workload", workload, "--gpus", str(n), "--warmup", str(warmup),
            "--impl", impl, "--no-cpu-baseline"]
    if steps is not None:
        args += ["--steps", str(steps)]
    if n == 1:
        return [sys.executable] + args
    # Rendezvous on the loopback address; an outer timeout bounds a hung rank.
    return (["timeout", "-k", "60", str(int(timeout)), sys.executable, "-m",
             "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
             "--master-addr", "127.0.0.1", "--master-port", str(free_port())] + args)


def run_bench(command, timeout, log_path):
    """Run one benchmark process; return its last JSON line (dict)."""
    with open(log_path, "w") as log:
        try:
            proc = subprocess.run(command, cwd=REPO, stdout=subprocess.PIPE, stderr=log,
                                  text=True, timeout=timeout + 90)
        except subprocess.TimeoutExpired as exc:
            raise ConfirmationError(f"benchmark timed out after {timeout} s") from exc
        log.write(proc.stdout)
    if proc.returncode:
        raise ConfirmationError(f"benchmark exited {proc.returncode}; see {log_path}")
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip().startswith("{")]
    if not lines:
        raise ConfirmationError(f"benchmark printed no JSON line; see {log_path}")
    return json.loads(lines[-1])


def check_line(line, workload_name, n, impl, mode):
    """A run enters a pair only if its JSON line is complete and describes this arm."""
    if line.get("unavailable"):
        raise ConfirmationError(f"arm unavailable: {line['unavailable']}")
    value = line.get("value")
    if type(value) not in (int, float) or not math.isfinite(value) or value <= 0:
        raise ConfirmationError("non-positive or non-finite value")
    if line.get("n_gpus") != n or (impl == "reference") != (line.get("impl") == "reference"):
        raise ConfirmationError("JSON line describes another arm")
    workload = (line.get("config") or {}).get("workload", "")
    if not workload:
        raise ConfirmationError("JSON line names no workload")
    if impl == "ours":
        reasons = (line.get("clocks") or {}).get("reasons") or []
        if any(r in REJECTED_REASONS for r in reasons):
            raise ConfirmationError(f"throttled run rejected ({', '.join(reasons)})")
        if mode == "cpu":
            e2e = (line.get("e2e") or {}).get("value")
            if type(e2e) not in (int, float) or not math.isfinite(e2e) or e2e <= 0:
                raise ConfirmationError("missing end-to-end value")


def pair_ratio(mode, pair):
    if mode == "gpus":
        return pair["many"]["value"] / pair["one"]["value"]
    return pair["ours"]["e2e"]["value"] / pair["reference"]["value"]


def summarize(mode, gpus, pairs):
    ratios = [pair_ratio(mode, p) for p in pairs]
    low, high = bootstrap_interval(ratios)
    out = {
        "paired_repetitions": len(pairs),
        "median_paired_ratio": statistics.median(ratios),
        "paired_ratios": ratios,
        "ci95_low": low,
        "ci95_high": high,
        "interval_method": INTERVAL_METHOD,
    }
    if mode == "gpus":
        out["ratio"] = f"value({gpus} GPUs) / value(1 GPU)"
        out["median_scaling_efficiency"] = statistics.median(ratios) / gpus
        out["scope"] = "One workload on one node and session; efficiency = ratio / G"
    else:
        out["ratio"] = "GPU end-to-end rate (host buffers) / reference CPU rate"
        out["scope"] = "One workload on one node and session; CPU = the host cores of that node"
    return out


def pairs_csv(mode, pairs):
    buffer = io.StringIO(newline="")
    out = csv.writer(buffer, lineterminator="\n")
    a, b = ("one", "many") if mode == "gpus" else ("reference", "ours")
    out.writerow(["repetition", "first", f"{a}_value", f"{b}_value", "ratio"])
    for pair in pairs:
        out.writerow([pair["repetition"], pair["order"][0], pair[a]["value"], pair[b]["value"],
                      pair_ratio(mode, pair)])
    return buffer.getvalue()


def receipt(output):
    return {name: hashlib.sha256((Path(output) / name).read_bytes()).hexdigest() for name in FILES}


def verify_scaling(output):
    """Recompute plan conformance, summary, CSV and receipt from the files (no CUDA)."""
    output = Path(output)
    report = json.loads((output / "scaling.json").read_text())
    mode, gpus = report["mode"], report["gpus"]
    plan = make_plan(mode, gpus, report["repetitions"])
    if (report.get("schema_version") != 1 or report.get("status") != "complete"
            or report.get("protocol") != PROTOCOL or report.get("plan") != plan
            or len(report["pairs"]) != len(plan)):
        raise ConfirmationError("scaling report provenance or completeness mismatch")
    workload = None
    for pair, planned in zip(report["pairs"], plan):
        if pair["order"] != planned["order"] or pair["repetition"] != planned["repetition"]:
            raise ConfirmationError("pair order differs from the plan")
        for arm in planned["order"]:
            n, impl = arm_spec(mode, arm, gpus)
            check_line(pair[arm], report["workload"], n, impl, mode)
        names = {pair[arm]["config"]["workload"] for arm in planned["order"]}
        if mode == "gpus" and len(names) != 1:
            raise ConfirmationError("the two arms of a pair ran different workloads")
        workload = workload or names
        if names != workload:
            raise ConfirmationError("pairs ran different workloads")
    if report.get("summary") != summarize(mode, gpus, report["pairs"]):
        raise ConfirmationError("summary differs from the paired evidence")
    if (output / "pairs.csv").read_text() != pairs_csv(mode, report["pairs"]):
        raise ConfirmationError("pairs.csv differs from the paired evidence")
    if json.loads((output / "receipt.json").read_text()) != receipt(output):
        raise ConfirmationError("receipt mismatch")
    return report["summary"]


def confirm_scaling(workload, output, mode="gpus", gpus=2, repetitions=3, steps=None, warmup=3,
                    timeout=600, dry_run=False, runner=None):
    """Run the paired plan; ``runner(command, timeout, log_path) -> dict`` defaults to a
    fresh benchmark process per run."""
    plan = make_plan(mode, gpus, repetitions)
    if not math.isfinite(timeout) or timeout <= 0 or warmup < 3:
        raise ConfirmationError("invalid timeout or warm-up (warm-up must be >= 3)")
    commands = {}
    for arm in plan[0]["order"]:
        n, impl = arm_spec(mode, arm, gpus)
        commands[arm] = bench_command(workload, n, impl, steps, warmup, timeout)
    if dry_run:
        return {"plan": plan, "commands": {k: " ".join(map(str, v)) for k, v in commands.items()},
                "timeout_sum_s": 2 * repetitions * timeout}
    output = Path(output)
    if output.exists():
        raise ConfirmationError("use a new output directory")
    runner = runner or run_bench
    output.mkdir(parents=True)
    (output / "logs").mkdir()
    report = {
        "schema_version": 1, "status": "running", "protocol": PROTOCOL, "mode": mode,
        "gpus": gpus, "workload": workload, "repetitions": repetitions, "steps": steps,
        "warmup": warmup, "timeout_s": timeout, "code_fingerprint": code_fingerprint(),
        "environment": environment(), "plan": plan, "pairs": [], "summary": None,
    }
    started = time.perf_counter()
    try:
        _atomic_json(output / "scaling.json", report)
        for planned in plan:
            pair = {"repetition": planned["repetition"], "order": planned["order"]}
            for arm in planned["order"]:
                n, impl = arm_spec(mode, arm, gpus)
                # A fresh port per multi-GPU run.
                cmd = bench_command(workload, n, impl, steps, warmup, timeout)
                line = runner(cmd, timeout, output / "logs" / f"rep{planned['repetition']}-{arm}.log")
                check_line(line, workload, n, impl, mode)
                pair[arm] = line
            report["pairs"].append(pair)
            _atomic_json(output / "scaling.json", report)
        report["status"] = "complete"
        report["summary"] = summarize(mode, gpus, report["pairs"])
        (output / "pairs.csv").write_text(pairs_csv(mode, report["pairs"]))
    except BaseException as exc:
        report["status"] = "interrupted" if isinstance(exc, KeyboardInterrupt) else "failed"
        report["summary"] = None
        report["error"] = f"{type(exc).__name__}: {exc}"
        raise
    finally:
        report["elapsed_s"] = time.perf_counter() - started
        _atomic_json(output / "scaling.json", report)
    _atomic_json(output / "receipt.json", receipt(output))
    verify_scaling(output)
    return report


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--workload", default="rmsnorm")
    parser.add_argument("--mode", choices=("gpus", "cpu"), default="gpus")
    parser.add_argument("--gpus", type=int, default=2)
    parser.add_argument("--repetitions", type=int, default=3)
    parser.add_argument("--steps", type=int, default=None)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--timeout", type=float, default=600)
    parser.add_argument("--output", type=Path)
    parser.add_argument("--dry-run", action="store_true")
    parser.add_argument("--verify", type=Path, help="verify a scaling directory (no CUDA)")
    args = parser.parse_args(argv)
    try:
        if args.verify:
            result = verify_scaling(args.verify)
        else:
            if args.output is None and not args.dry_run:
                raise ConfirmationError("--output is required")
            result = confirm_scaling(args.workload, args.output, args.mode, args.gpus,
                                     args.repetitions, args.steps, args.warmup, args.timeout,
                                     args.dry_run)
            if not args.dry_run:
                result = result["summary"]
        print(json.dumps(result, indent=2, allow_nan=False))
        return 0
    except (ValueError, RuntimeError, OSError, KeyError, TypeError) as exc:
        print(f"Scaling confirmation failed: {exc}")
        return 1


if __name__ == "__main__":
    os.environ.setdefault("PYTHONUNBUFFERED", "1")
    raise SystemExit(main())

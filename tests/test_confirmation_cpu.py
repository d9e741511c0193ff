"""Paired confirmation (single GPU, candidate vs torch) and paired scaling
confirmation (1 vs G GPUs, CPU reference vs GPU) on the host: the GPU work is
replaced by injected fakes, everything else (plans, validation, statistics,
evidence files, receipts, verification) is the real code."""

import json
import shutil

import pytest

from flashattentionanycard_b200.configs.search_spaces import Workload
from flashattentionanycard_b200.tuner import confirmation as conf
from flashattentionanycard_b200.tuner import scaling
from flashattentionanycard_b200.tuner.engine import run_search
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

MEAS = Measurement(warmup=1, repeats=3, batch=1, validation_seeds=2)
HW = Hardware("B200 test double", (10, 0), 148, 180 * 1024**3, 227 * 1024, uuid="GPU-test-0")


def timing(implementation, latency=1.0, dtype="bf16", repeats=3):
    samples = [latency * (1 + 0.01 * i) for i in range(repeats)]
    out = sample_statistics(samples)
    rtol, atol = TOLERANCES[dtype]
    out.update(status="ok", implementation=implementation, protocol=MEASUREMENT_PROTOCOL,
               precision_policy=PRECISION_POLICY,
               validation=[{"max_abs_error": 0.01, "rtol": rtol, "atol": atol}] * 2)
    return out


@pytest.fixture
def source(tmp_path):
    workload = Workload("rmsnorm", 64, 256, dtype="bf16")
    space = {"ROWS_PER_CTA": [1, 2], "num_warps": [4, 8], "num_stages": [1]}

    def evaluator(params):
        return timing(CANDIDATE, 0.01 * params["ROWS_PER_CTA"] + 0.001 * params["num_warps"])

    run_search(workload, HW, space, "grid", 0, 4, tmp_path / "search", measurement=MEAS,
               evaluator=evaluator)
    return tmp_path / "search" / "result.json"


def fake_pair(candidate_ms=1.0, torch_ms=2.0, hw=HW):
    def evaluate_pair(workload, hardware, params, measurement, timeout, log_dir, number, *,
                      order):
        return {"status": "ok", "order": order, "data_seed": workload.data_seed,
                "candidate": timing(CANDIDATE, candidate_ms * (1 + 0.02 * number)),
                "torch": timing(BASELINES[workload.kernel], torch_ms),
                "hardware": hw.to_dict()}
    return evaluate_pair


@pytest.fixture
def detect(monkeypatch):
    monkeypatch.setattr(conf.Hardware, "detect", classmethod(lambda cls, device=0: HW))


def test_plan_uses_held_out_seeds_and_balanced_order(source):
    _, workload, measurement = conf.freeze_source(source.read_bytes())
    plan = conf.make_plan(workload, measurement, 6)
    search_seeds = {workload.data_seed + i for i in range(measurement.validation_seeds)}
    seeds = [p["data_seed"] for p in plan]
    assert len(set(seeds)) == 6 and not search_seeds & set(seeds)
    firsts = [p["order"][0] for p in plan]
    assert firsts.count("candidate") == firsts.count("torch") == 3
    with pytest.raises(conf.ConfirmationError):
        conf.make_plan(workload, measurement, 2)


def test_confirm_and_verify(source, tmp_path, detect):
    out = tmp_path / "confirm"
    report = conf.confirm(source, out, repetitions=4, evaluate_pair=fake_pair())
    summary = report["summary"]
    assert summary["paired_repetitions"] == 4
    assert 1.85 < summary["median_paired_speedup"] < 2.0
    assert summary["ci95_low"] <= summary["median_paired_speedup"] <= summary["ci95_high"]
    assert conf.verify_confirmation(out) == summary
    assert conf.main(["--verify", str(out)]) == 0


def test_dry_run_needs_no_device(source, tmp_path):
    plan = conf.confirm(source, tmp_path / "never", repetitions=3, dry_run=True)
    assert plan["baseline"] == BASELINES["rmsnorm"] and len(plan["plan"]) == 3
    assert not (tmp_path / "never").exists()


@pytest.mark.parametrize("mutation", ["fingerprint", "winner", "samples", "counts", "protocol"])
def test_invalid_source_is_rejected(source, tmp_path, mutation):
    data = json.loads(source.read_text())
    if mutation == "fingerprint":
        data["metadata"]["code_fingerprint"] = "0" * 64
    elif mutation == "winner":
        data["best"] = next(t for t in data["trials"] if t != data["best"])
    elif mutation == "samples":
        data["best"]["attrs"]["measurement"]["samples_ms"][0] *= 2
    elif mutation == "counts":
        data["attempts"] += 1
    else:
        data["metadata"]["protocol"] = "other"
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps(data))
    with pytest.raises(conf.ConfirmationError):
        conf.confirm(bad, tmp_path / "out", repetitions=3, dry_run=True)


@pytest.mark.parametrize("failure", [RuntimeError("worker_timeout"), KeyboardInterrupt()])
def test_failure_keeps_partial_pairs_and_no_speedup(source, tmp_path, detect, failure):
    good = fake_pair()

    def flaky(*args, number, **kw):
        if number == 2:
            raise failure
        return good(*args, number=number, **kw)

    def evaluate_pair(workload, hardware, params, measurement, timeout, log_dir, number, *, order):
        return flaky(workload, hardware, params, measurement, timeout, log_dir, number=number,
                     order=order)

    out = tmp_path / "confirm"
    with pytest.raises(type(failure)):
        conf.confirm(source, out, repetitions=4, evaluate_pair=evaluate_pair)
    report = json.loads((out / "confirmation.json").read_text())
    assert report["status"] in ("failed", "interrupted") and report["summary"] is None
    assert len(report["pairs"]) == 2 and not (out / "receipt.json").exists()


@pytest.mark.parametrize("mutation", ["speedup", "csv", "order", "hardware"])
def test_tampering_is_detected(source, tmp_path, detect, mutation):
    out = tmp_path / "confirm"
    conf.confirm(source, out, repetitions=3, evaluate_pair=fake_pair())
    report = json.loads((out / "confirmation.json").read_text())
    if mutation == "speedup":
        report["summary"]["median_paired_speedup"] *= 1.5
    elif mutation == "order":
        report["pairs"][0]["order"].reverse()
    elif mutation == "hardware":
        report["pairs"][1]["hardware"]["uuid"] = "GPU-other"
    if mutation == "csv":
        (out / "pairs.csv").write_text((out / "pairs.csv").read_text().replace(",", ";", 3))
    else:
        (out / "confirmation.json").write_text(json.dumps(report))
    with pytest.raises(conf.ConfirmationError):
        conf.verify_confirmation(out)


def test_other_device_or_overwrite_rejected(source, tmp_path, monkeypatch):
    other = Hardware("B200 test double", (10, 0), 148, 180 * 1024**3, 227 * 1024,
                     uuid="GPU-test-1")
    monkeypatch.setattr(conf.Hardware, "detect", classmethod(lambda cls, device=0: other))
    with pytest.raises(conf.ConfirmationError, match="GPU"):
        conf.confirm(source, tmp_path / "a", repetitions=3, evaluate_pair=fake_pair())
    (tmp_path / "b").mkdir()
    with pytest.raises(conf.ConfirmationError, match="new"):
        conf.confirm(source, tmp_path / "b", repetitions=3, evaluate_pair=fake_pair())


def test_bootstrap_resamples_pairs():
    low, high = conf.bootstrap_interval([2.0, 2.0, 2.0])
    assert low == high == 2.0
    low, high = conf.bootstrap_interval([1.0, 2.0, 3.0, 4.0])
    assert 1.0 <= low < high <= 4.0
    assert conf.bootstrap_interval([1.0, 2.0, 3.0, 4.0]) == (low, high)  # seeded


# ------------------------------------------------------------------ scaling
def fake_bench(values, reasons=(), unavailable=False):
    """runner(command, timeout, log_path) answering like bench.py's JSON line."""
    calls = []

    def runner(command, timeout, log_path):
        n = int(command[command.index("--gpus") + 1])
        impl = command[command.index("--impl") + 1]
        calls.append((n, impl, command))
        if impl == "reference":
            if unavailable:
                return {"impl": "reference", "unavailable": "not here"}
            return {"impl": "reference", "value": values["reference"], "n_gpus": 1,
                    "config": {"workload": "rmsnorm_bf16_4096x4096_eps1e-6"}}
        v = values[n] * (1 + 0.01 * len(calls))
        return {"impl": "ours", "value": v, "n_gpus": n,
                "e2e": {"value": values.get("e2e", v / 10)},
                "config": {"workload": "rmsnorm_bf16_4096x4096_eps1e-6"},
                "clocks": {"reasons": list(reasons)}}

    runner.calls = calls
    return runner


def test_scaling_gpus_mode_pairs_and_verifies(tmp_path):
    runner = fake_bench({1: 5000.0, 4: 19000.0})
    out = tmp_path / "scale"
    report = scaling.confirm_scaling("rmsnorm", out, "gpus", 4, 4, runner=runner)
    s = report["summary"]
    assert s["paired_repetitions"] == 4 and 3.5 < s["median_paired_ratio"] < 4.0
    assert s["median_scaling_efficiency"] == pytest.approx(s["median_paired_ratio"] / 4)
    firsts = [c[0] for c in runner.calls[::2]]
    assert firsts == [1, 4, 1, 4]  # balanced order
    multi = [c[2] for c in runner.calls if c[0] == 4]
    assert all("torch.distributed.run" in c and "127.0.0.1" in c and c[0] == "timeout"
               for c in multi)
    assert scaling.verify_scaling(out) == s
    assert scaling.main(["--verify", str(out)]) == 0
    report_path = out / "scaling.json"
    data = json.loads(report_path.read_text())
    data["pairs"][1]["many"]["value"] *= 2
    report_path.write_text(json.dumps(data))
    with pytest.raises(conf.ConfirmationError):
        scaling.verify_scaling(out)


def test_scaling_cpu_mode_uses_end_to_end_rate(tmp_path):
    runner = fake_bench({1: 5000.0, "reference": 9.0, "e2e": 90.0})
    report = scaling.confirm_scaling("rmsnorm", tmp_path / "cpu", "cpu", repetitions=3,
                                     runner=runner)
    assert report["summary"]["median_paired_ratio"] == pytest.approx(10.0)
    assert {c[1] for c in runner.calls} == {"reference", "ours"}
    shutil.copy(tmp_path / "cpu" / "pairs.csv", tmp_path / "copy.csv")
    assert scaling.verify_scaling(tmp_path / "cpu")["median_paired_ratio"] == pytest.approx(10.0)


@pytest.mark.parametrize("case", ["throttled", "unavailable"])
def test_scaling_rejects_bad_runs(tmp_path, case):
    runner = (fake_bench({1: 1.0, 2: 2.0}, reasons=["hw_thermal_slowdown"]) if case == "throttled"
              else fake_bench({1: 1.0, "reference": 1.0}, unavailable=True))
    mode = "gpus" if case == "throttled" else "cpu"
    out = tmp_path / case
    with pytest.raises(conf.ConfirmationError):
        scaling.confirm_scaling("rmsnorm", out, mode, 2, 3, runner=runner)
    report = json.loads((out / "scaling.json").read_text())
    assert report["status"] == "failed" and report["summary"] is None


def test_scaling_dry_run_and_plan_rules(tmp_path):
    dry = scaling.confirm_scaling("gemm8192", tmp_path / "x", "gpus", 8, 3, dry_run=True)
    assert "--nproc-per-node=8" in dry["commands"]["many"]
    assert dry["commands"]["one"].split()[1] == "bench.py"
    assert not (tmp_path / "x").exists()
    with pytest.raises(conf.ConfirmationError):
        scaling.make_plan("gpus", 1, 3)
    with pytest.raises(conf.ConfirmationError):
        scaling.make_plan("cpu", 1, 2)

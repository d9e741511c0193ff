"""Search engine, warm-start transfer and CLI (no GPU): mirrors the reference's
tests/test_engine.py, with the evaluator injected and subprocess.run faked."""

from flashattentionanycard_b200.tuner.engine import warm_start

import json
import subprocess
import time

import pytest

from flashattentionanycard_b200.configs.search_spaces import Workload, search_space
from flashattentionanycard_b200.tuner import engine
from flashattentionanycard_b200.tuner.engine import EvaluationFailure, run_search
from flashattentionanycard_b200.tuner.hardware import Hardware
from flashattentionanycard_b200.tuner.worker import Measurement

SPACE = {"ROWS_PER_CTA": [1, 2], "num_warps": [4, 8]}


def objective(p):
    return {"latency_ms": float(p["ROWS_PER_CTA"] + p["num_warps"])}


def search(tmp_path, hardware, method="grid", budget=4, evaluator=objective, space=SPACE, **kw):
    return run_search(Workload("rmsnorm"), hardware, space, method, 0, budget, tmp_path,
                      evaluator=evaluator, startup_trials=2, **kw)


@pytest.mark.parametrize("method", ["grid", "random"])
def test_attempt_accounting_and_persistence(tmp_path, hardware, method):
    result = search(tmp_path, hardware, method)
    assert result["attempts"] == result["successful_evaluations"] == 4
    assert result["best"]["value"] >= 5
    assert json.loads((tmp_path / "result.json").read_text()) == result
    assert (tmp_path / "trials.csv").read_text().count("\n") == 5
    assert all(t["attrs"]["elapsed_s"] > 0 for t in result["trials"])
    assert result["metadata"]["code_fingerprint"] == engine.code_fingerprint()


def test_grid_exhaustion(tmp_path, hardware):
    result = search(tmp_path, hardware, "grid", 100)
    assert result["attempts"] == result["unique_successful_configs"] == 4
    assert result["best"]["value"] == 5.0


def test_random_shares_grid_sized_budget_cap(tmp_path, hardware):
    result = search(tmp_path, hardware, "random", 100)
    assert result["attempts"] == result["metadata"]["budget"] == 4
    assert result["metadata"]["requested_budget"] == 100


def test_no_silent_failures(tmp_path, hardware):
    def fail(p):
        raise EvaluationFailure("simulated timeout")

    result = search(tmp_path, hardware, evaluator=fail)
    assert result["status"] == "failed" and result["best"] is None
    assert all(t["state"] == "FAIL" and "failure" in t["attrs"] for t in result["trials"])


@pytest.mark.parametrize("value", [float("nan"), float("inf"), 0, -1])
def test_reject_nonpositive_or_nonfinite_measurement(tmp_path, hardware, value):
    result = search(tmp_path, hardware, budget=1, evaluator=lambda p: {"latency_ms": value})
    assert result["status"] == "failed"


def test_pruning_counts_toward_budget(tmp_path, hardware):
    space = {"ROWS_PER_CTA": [1], "num_warps": [64]}
    result = run_search(Workload("rmsnorm"), hardware, space, "grid", 1, 5, tmp_path,
                        evaluator=lambda p: pytest.fail("Pruned config must not execute"))
    assert result["attempts"] == 1
    assert result["trials"][0]["state"] == "PRUNED"
    assert result["trials"][0]["attrs"]["prune_reason"] == "illegal_threads_per_block"


def test_gemm_space_prunes_shared_memory_overflow(tmp_path, hardware):
    space = {"BLOCK_M": [128], "BLOCK_N": [256], "BLOCK_K": [64], "num_warps": [6],
             "num_stages": [4, 6], "GROUP_M": [8]}
    result = run_search(Workload("gemm"), hardware, space, "grid", 0, 2, tmp_path,
                        evaluator=lambda p: {"latency_ms": 1.0})
    states = {t["params"]["num_stages"]: t["state"] for t in result["trials"]}
    assert states == {4: "COMPLETE", 6: "PRUNED"}


def test_unexpected_bug_aborts_with_checkpoint(tmp_path, hardware):
    def fail(p):
        raise KeyError("programming bug")

    with pytest.raises(KeyError):
        search(tmp_path, hardware, evaluator=fail)
    assert json.loads((tmp_path / "result.json").read_text())["status"] == "interrupted"


def test_refuse_overwrite(tmp_path, hardware):
    (tmp_path / "important.txt").write_text("retain")
    with pytest.raises(ValueError, match="empty"):
        search(tmp_path, hardware)
    assert (tmp_path / "important.txt").read_text() == "retain"


def test_tpe_needs_optuna_or_runs(tmp_path, hardware):
    if engine.have_optuna():
        result = search(tmp_path, hardware, "tpe")
        assert result["attempts"] == 4
    else:
        with pytest.raises(RuntimeError, match="optuna"):
            search(tmp_path, hardware, "tpe")


def test_transfer_compatibility_and_pruning(tmp_path, hardware):
    search(tmp_path / "source", hardware, "grid")
    path = tmp_path / "source/result.json"
    queue, provenance = warm_start(path, Workload("rmsnorm"), SPACE, 2, hardware, lambda p: None)
    assert queue[0] == {"ROWS_PER_CTA": 1, "num_warps": 4} and len(queue) == 2
    assert provenance["strategy"] == "ranked_parameters_remeasured_on_target"
    with pytest.raises(ValueError, match="mismatch"):
        warm_start(path, Workload("rmsnorm", n=7), SPACE, 2, hardware, lambda p: None)
    with pytest.raises(ValueError, match="No legal"):
        warm_start(path, Workload("rmsnorm"), SPACE, 2, hardware, lambda p: "illegal")
    with pytest.raises(ValueError, match="top_k"):
        warm_start(path, Workload("rmsnorm"), SPACE, 0, hardware, lambda p: None)
    data = json.loads(path.read_text())
    data["metadata"]["code_fingerprint"] = "stale"
    path.write_text(json.dumps(data))
    with pytest.raises(ValueError, match="different kernel code"):
        warm_start(path, Workload("rmsnorm"), SPACE, 2, hardware, lambda p: None)


def test_fingerprint_covers_cuda_sources(tmp_path, monkeypatch):
    pkg = tmp_path / "pkg"
    for sub in ("kernels", "configs", "tuner", "csrc"):
        (pkg / sub).mkdir(parents=True)
    (tmp_path / "include").mkdir()
    (pkg / "csrc" / "k.cuh").write_text("// v1")
    (tmp_path / "include" / "a.h").write_text("int f(void);")
    monkeypatch.setattr(engine, "PACKAGE", pkg)
    first = engine.code_fingerprint()
    (pkg / "csrc" / "k.cuh").write_text("// v2")
    second = engine.code_fingerprint()
    (tmp_path / "include" / "a.h").write_text("int f(int);")
    assert len({first, second, engine.code_fingerprint()}) == 3


def test_isolated_timeout_and_crash(tmp_path, hardware, monkeypatch):
    def timeout(*args, **kwargs):
        raise subprocess.TimeoutExpired("worker", 1)

    monkeypatch.setattr(subprocess, "run", timeout)
    with pytest.raises(EvaluationFailure, match="timeout"):
        engine.isolated_evaluate(Workload(), hardware, {}, Measurement(), 1, tmp_path, 0)
    monkeypatch.setattr(subprocess, "run", lambda *a, **kw: subprocess.CompletedProcess([], -11))
    with pytest.raises(EvaluationFailure, match="exit_-11"):
        engine.isolated_evaluate(Workload(), hardware, {}, Measurement(), 1, tmp_path, 1)


def test_isolated_worker_error_is_a_failure(tmp_path, hardware):
    """A real worker process on a CPU-only machine: the worker reports the
    error in its JSON and the engine turns it into EvaluationFailure."""
    with pytest.raises(EvaluationFailure):
        engine.isolated_evaluate(Workload("rmsnorm", 4, 16), hardware, {}, Measurement(), 120,
                                 tmp_path, 0)
    assert (tmp_path / "trial-0.log").exists()


def test_wall_budget_stops_after_attempt(tmp_path, hardware):
    def slow(p):
        time.sleep(0.04)
        return objective(p)

    space = {"ROWS_PER_CTA": [1, 2, 4, 8], "num_warps": [1, 2, 4, 8, 16]}
    result = search(tmp_path, hardware, budget=100, evaluator=slow, space=space, time_budget=0.2)
    assert result["attempts"] < 20


def test_cli_dry_run_and_invalid_options(tmp_path, capsys):
    rc = engine.main(["--dry-run", "--kernel", "moe_grouped_gemm", "--output",
                      str(tmp_path / "unused")])
    assert rc == 0 and not (tmp_path / "unused").exists()
    plan = json.loads(capsys.readouterr().out.strip().splitlines()[0])
    assert plan["workload"]["kernel"] == "moe_grouped_gemm" and plan["grid_size"] > 0
    assert engine.main(["--dry-run", "--expert-tokens", "0,0", "--kernel", "moe_grouped_gemm",
                        "--output", str(tmp_path / "x")]) == 2
    assert engine.main(["--dry-run", "--warm-start", "r.json", "--output", str(tmp_path)]) == 2


def test_hardware_detect_requires_sm100_double():
    hw = Hardware("CPU test double", (10, 0), 148, 1, 1)
    assert hw.to_dict()["capability"] == [10, 0]

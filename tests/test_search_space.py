"""CPU legality tests, mirroring the reference's tests/test_correctness.py:16-55."""

import pytest

from flashattentionanycard_b200.configs.search_spaces import (
    Workload,
    default_params,
    grid_configs,
    grid_size,
    search_space,
    validate_params,
)
from flashattentionanycard_b200.tuner.hardware import (
    Hardware,
    gemm_pair_shared_bytes,
    gemm_shared_bytes,
    nvlink_topology,
    parse_topology,
    prune_reason,
    resource_estimate,
)


@pytest.mark.parametrize("kernel", ["gemm", "rmsnorm", "moe_grouped_gemm"])
@pytest.mark.parametrize("profile", ["full", "smoke"])
def test_shared_search_domain(kernel, profile):
    space = search_space(kernel, profile)
    configs = list(grid_configs(space))
    assert len(configs) == grid_size(space)
    assert len({tuple(p.items()) for p in configs}) == len(configs)
    assert all(validate_params(p, space) for p in configs)
    assert validate_params(default_params(kernel), search_space(kernel))


def test_hard_legality_and_heuristics_are_distinct(hardware):
    p = next(grid_configs(search_space("gemm")))
    p.update(BLOCK_N=128, num_stages=6)
    assert resource_estimate("gemm", p)["shared_bytes_estimate"] <= hardware.shared_memory_per_block
    assert prune_reason(hardware, "gemm", p) is None
    assert prune_reason(hardware, "gemm", p, heuristic_smem=True) == "heuristic_shared_memory_estimate"
    p.update(BLOCK_N=256, num_stages=5)  # 5 x 48 KB ring: does not fit
    assert prune_reason(hardware, "gemm", p) == "shared_memory_exceeds_device_limit"
    p["num_warps"] = 64
    assert prune_reason(hardware, "gemm", p) == "illegal_threads_per_block"
    p["num_warps"] = 4
    assert prune_reason(hardware, "gemm", p) == "illegal_threads_per_block"


def test_every_full_space_config_is_classified(hardware):
    for kernel in ("gemm", "moe_grouped_gemm"):
        legal = [p for p in grid_configs(search_space(kernel)) if prune_reason(hardware, kernel, p) is None]
        assert legal, kernel
        for p in legal:
            experts = 64 if kernel == "moe_grouped_gemm" else 0
            if p.get("CTA_GROUP", 1) == 2:
                assert gemm_pair_shared_bytes(p["BLOCK_N"], p["num_stages"], experts) <= 227 * 1024
            else:
                assert gemm_shared_bytes(p["BLOCK_N"], p["num_stages"], 64) <= 227 * 1024
        assert any(p["CTA_GROUP"] == 2 for p in legal)


def test_rmsnorm_limit(hardware):
    assert prune_reason(hardware, "rmsnorm", {"ROWS_PER_CTA": 8, "num_warps": 4}, 4096) is None
    assert prune_reason(hardware, "rmsnorm", {"ROWS_PER_CTA": 4, "num_warps": 64}, 4097)
    est = resource_estimate("rmsnorm", {"ROWS_PER_CTA": 1, "num_warps": 4}, 4096)
    assert est["threads_per_row"] == 128 and est["vectors_per_thread"] == 4


@pytest.mark.parametrize(
    "kwargs",
    [
        {"m": 0},
        {"dtype": "fp32"},
        {"kernel": "bad"},
        {"expert_tokens": (0, 0)},
        {"expert_tokens": (-1, 2)},
        {"epsilon": float("nan")},
        {"data_seed": -1},
    ],
)
def test_invalid_workload(kwargs):
    with pytest.raises(ValueError):
        Workload(**kwargs)


TOPO = """\
\tGPU0\tGPU1\tGPU2\tNIC0\tCPU Affinity\tNUMA Affinity
GPU0\t X \tNV18\tNV18\tSYS\t0-55\t0
GPU1\tNV18\t X \tNV18\tSYS\t0-55\t0
GPU2\tNV18\tNV18\t X \tSYS\t56-111\t1
NIC0\tSYS\tSYS\tSYS\t X
"""


def test_topology_header_with_terminal_escapes():
    """nvidia-smi prints the header row underlined (ESC[4m ... ESC[0m)."""
    text = ("\t\x1b[4mGPU0\tGPU1\tCPU Affinity\tNUMA Affinity\tGPU NUMA ID\x1b[0m\n"
            "GPU0\t X \tNV18\t0-55\t0\t\tN/A\n"
            "GPU1\tNV18\t X \t0-55\t0\t\tN/A\n")
    topo = parse_topology(text)
    assert topo == {0: {0: "X", 1: "NV18"}, 1: {0: "NV18", 1: "X"}}

    class Fake:
        stdout = text

    view = nvlink_topology(0, runner=lambda *a, **k: Fake())
    assert view == {"gpus": 2, "peers": {"1": {"link": "NV18", "nvlinks": 18}},
                    "all_nvlink": True}


def test_topology_parsing_with_fake_nvidia_smi():
    topo = parse_topology(TOPO)
    assert topo[0][1] == "NV18" and topo[2][0] == "NV18" and topo[1][1] == "X"

    class Fake:
        stdout = TOPO

    view = nvlink_topology(1, runner=lambda *a, **k: Fake())
    assert view["gpus"] == 3 and view["all_nvlink"]
    assert view["peers"]["0"] == {"link": "NV18", "nvlinks": 18}

    def missing(*a, **k):
        raise OSError("no nvidia-smi")

    assert nvlink_topology(0, runner=missing) == {}


def test_hardware_dict_roundtrip(hardware):
    d = hardware.to_dict()
    assert d["capability"] == [10, 0] and d["sm_count"] == 148
    assert Hardware("x", (10, 0), 1, 1, 1) == Hardware("x", (10, 0), 1, 1, 1, nvlink={"a": 1})

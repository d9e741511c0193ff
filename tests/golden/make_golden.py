"""Regenerate the golden fixtures from the reference implementation itself.

Runs only where the reference checkout is present (the build container); the
committed ``*.npz`` files are what the tests read.  Usage:

    python tests/golden/make_golden.py PATH_TO_REFERENCE_CHECKOUT

For every case it records:
  * the inputs (16-bit storage bits), drawn exactly as the reference's
    ``worker.prepare`` draws them but from a CPU generator;
  * ``ref``: the reference's own FP32 reference from ``worker.prepare(...,
    device=cpu, implementation="torch")`` (bo_kernel_tuner/tuner/worker.py:45-105);
  * ``triton``: the output of the reference's Triton kernel run on the CPU by
    Triton's interpreter (TRITON_INTERPRET=1), with the first configuration of
    the reference's smoke search space.  The interpreter's bf16 ``tl.dot`` is
    not usable, so bf16 GEMM / grouped GEMM cases carry ``ref`` only.
Routing cases (no reference implementation) carry numpy's stable argsort,
bincount and cumsum of seeded Zipf top-2 expert ids.
"""

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def bits(t):
    import torch

    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main(reference_root):
    sys.path.insert(0, reference_root)
    sys.path.insert(0, REPO)
    import torch
    from bo_kernel_tuner.configs.search_spaces import Workload as RefWorkload
    from bo_kernel_tuner.configs.search_spaces import grid_configs, search_space
    from bo_kernel_tuner.kernels import gemm as ref_gemm
    from bo_kernel_tuner.kernels import moe_grouped_gemm as ref_moe
    from bo_kernel_tuner.kernels import rmsnorm as ref_rmsnorm
    from bo_kernel_tuner.tuner.worker import prepare as ref_prepare

    from flashattentionanycard_b200.configs.search_spaces import Workload
    from flashattentionanycard_b200.tuner.worker import generate_inputs, reference_output
    from flashattentionanycard_b200.workloads import zipf_routing

    torch.set_num_threads(1)
    cpu = torch.device("cpu")
    experts = (0, 1, 33, 0, 9)  # reference tests/test_correctness.py:563
    cases = {}

    def record(kernel, dtype, shape, seed, experts_used=experts):
        m, n, k = shape
        rw = RefWorkload(kernel, m, n, k, dtype, experts_used)
        _, _, ref = ref_prepare(rw, cpu, seed, 4, "torch")
        w = Workload(kernel, m, n, k, dtype, experts_used)
        inputs = generate_inputs(w, seed)
        mine = reference_output(w, inputs)
        if not torch.equal(mine, ref):
            raise SystemExit(f"input draw differs from the reference for {kernel} {shape} {seed}")
        key = f"{kernel}|{dtype}|{m}x{n}x{k}|{seed}"
        entry = {"ref": ref.numpy().astype(np.float32)}
        for name, value in inputs.items():
            entry[name] = bits(value) if hasattr(value, "view") else np.asarray(value, np.int64)
        params = next(grid_configs(search_space(kernel, "smoke")))
        interp_ok = dtype == "fp16" or kernel == "rmsnorm"
        if interp_ok:
            if kernel == "gemm":
                out = torch.full((m, n), float("nan"), dtype=inputs["a"].dtype)
                ref_gemm.launch(inputs["a"], inputs["b"], out, params)
            elif kernel == "rmsnorm":
                out = torch.full((m, n), float("nan"), dtype=inputs["x"].dtype)
                ref_rmsnorm.launch(inputs["x"], inputs["weight"], out, params, 1e-6)
            else:
                t = sum(experts_used)
                out = torch.full((t, n), float("nan"), dtype=inputs["x"].dtype)
                offsets = torch.tensor(inputs["starts"], dtype=torch.int64)
                ref_moe.launch(inputs["x"], inputs["weight"], offsets, out, params, 4)
            entry["triton"] = bits(out)
            entry["triton_params"] = np.asarray(sorted(params.items()), dtype=object).astype(str)
        cases[key] = entry

    for kernel in ("gemm", "rmsnorm", "moe_grouped_gemm"):
        for dtype in ("fp16", "bf16"):
            for shape, seeds in (((64, 128, 64), (0,)), ((37, 77, 93), (0, 17)), ((1, 1, 1), (0, 17))):
                for seed in seeds:
                    record(kernel, dtype, shape, seed)
    # The 127 x 193 x 257 bf16 smoke GEMM shape, seed 0, reference N(0,1) draw.
    record("gemm", "bf16", (127, 193, 257), 0)
    # Grouped GEMM with the reference smoke suite's expert counts (runpod/configs/smoke.json).
    record("moe_grouped_gemm", "fp16", (1, 64, 32), 0, (0, 1, 17, 65))

    flat = {}
    for key, entry in cases.items():
        for name, value in entry.items():
            flat[f"{key}|{name}"] = value
    np.savez_compressed(os.path.join(HERE, "reference_kernels.npz"), **flat)

    routing = {}
    for tokens, n_experts, seed in ((512, 64, 0), (1000, 8, 3), (4096 + 37, 64, 5)):
        ids = zipf_routing(tokens, n_experts, 2, 1.1, seed).numpy().reshape(-1)
        key = f"zipf|{tokens}|{n_experts}|{seed}"
        counts = np.bincount(ids, minlength=n_experts)
        routing[f"{key}|ids"] = ids.astype(np.int32)
        routing[f"{key}|counts"] = counts.astype(np.int32)
        routing[f"{key}|offsets"] = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
        routing[f"{key}|perm"] = np.argsort(ids, kind="stable").astype(np.int32)
    np.savez_compressed(os.path.join(HERE, "routing.npz"), **routing)
    print(f"{len(cases)} kernel cases, {len(routing) // 4} routing cases written to {HERE}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py PATH_TO_REFERENCE_CHECKOUT")
    main(sys.argv[1])

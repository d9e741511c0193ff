"""Run bo-kernel-tuner's own tuner plumbing on the sm_100a kernels.

The reference binds its hot path through five modules: the three kernels its
worker imports (``bo_kernel_tuner/tuner/worker.py:51-52``), the search space
(``configs/search_spaces.py``) and the legality checks (``tuner/hardware.py``)
that its engine prunes with.  Swapping exactly those five files for one-line
re-exports of this package makes the reference's unmodified worker (subprocess
isolation, FP32 gate, CUDA-graph measurement), engine, confirmation protocol
and tests drive these kernels.  ``overlay`` does that swap on a copy of the
reference package, leaving the original untouched:

    python -m flashattentionanycard_b200.dropin /path/containing/bo_kernel_tuner OUT_DIR
    PYTHONPATH=OUT_DIR:$PYTHONPATH python -m bo_kernel_tuner.run_benchmark ...

(the reference's ``run_benchmark`` and ``engine`` need Optuna installed).
"""

import shutil
import sys
from pathlib import Path

# Reference module (path inside the bo_kernel_tuner package) -> replacement source.
SHIMS = {
    "kernels/gemm.py": (
        '"""sm_100a tcgen05 GEMM (flashattentionanycard_b200), drop-in for the Triton kernel."""\n'
        "from flashattentionanycard_b200.kernels.gemm import launch  # noqa: F401\n"
    ),
    "kernels/rmsnorm.py": (
        '"""sm_100a RMSNorm (flashattentionanycard_b200), drop-in for the Triton kernel."""\n'
        "from flashattentionanycard_b200.kernels.rmsnorm import launch  # noqa: F401\n"
    ),
    "kernels/moe_grouped_gemm.py": (
        '"""sm_100a grouped GEMM (flashattentionanycard_b200), drop-in for the Triton kernel."""\n'
        "from flashattentionanycard_b200.kernels.moe_grouped_gemm import launch  # noqa: F401\n"
    ),
    "configs/search_spaces.py": (
        '"""Search domains over the sm_100a kernels\' CUDA launch parameters."""\n'
        "from flashattentionanycard_b200.configs.search_spaces import (  # noqa: F401\n"
        "    KERNELS, SPACE_VERSION, Workload, default_params, grid_configs, grid_size,\n"
        "    search_space, validate_params)\n"
    ),
    "tuner/hardware.py": (
        '"""sm_100 detection and legality checks of the sm_100a kernels."""\n'
        "from flashattentionanycard_b200.tuner.hardware import (  # noqa: F401\n"
        "    Hardware, nvlink_topology, prune_reason, resource_estimate)\n"
    ),
}


def reference_package(root):
    """The ``bo_kernel_tuner`` package directory under ``root`` (or ``root`` itself)."""
    root = Path(root)
    for candidate in (root / "bo_kernel_tuner", root):
        if (candidate / "tuner" / "worker.py").is_file() and (candidate / "kernels").is_dir():
            return candidate
    raise FileNotFoundError(f"no bo_kernel_tuner package under {root}")


def overlay(reference_root, out_dir):
    """Copy the reference package into ``out_dir`` with the five shims in place.

    Returns the directory to put on ``PYTHONPATH`` (it contains
    ``bo_kernel_tuner``)."""
    src = reference_package(reference_root)
    out_dir = Path(out_dir)
    dst = out_dir / "bo_kernel_tuner"
    if dst.exists():
        raise FileExistsError(f"{dst} exists; use a fresh directory")
    shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    for rel, text in SHIMS.items():
        (dst / rel).write_text(text)
    return out_dir


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2:
        print(__doc__)
        return 2
    print(overlay(argv[0], argv[1]))
    return 0


if __name__ == "__main__":
    sys.exit(main())

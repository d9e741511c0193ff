"""Helpers of the drop-in tests: where the reference package is, and the
environment in which its own modules import these kernels."""

import os
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
STUBS = Path(__file__).resolve().parent / "dropin_stubs"


def reference_root():
    """Directory holding the reference's bo_kernel_tuner package, or None:
    $BOKT_REFERENCE_PATH, else the offline install under baseline/_ref."""
    for candidate in (os.environ.get("BOKT_REFERENCE_PATH"), REPO / "baseline" / "_ref"):
        if candidate and (Path(candidate) / "bo_kernel_tuner" / "tuner" / "worker.py").is_file():
            return Path(candidate)
    return None


def overlay_env(overlay_dir):
    """Environment for a child process: the overlaid reference first, then the
    optuna stand-in and this repository."""
    env = dict(os.environ)
    parts = [str(overlay_dir), str(STUBS), str(REPO)]
    if env.get("PYTHONPATH"):
        parts.append(env["PYTHONPATH"])
    env["PYTHONPATH"] = os.pathsep.join(parts)
    return env

"""Access to the committed golden fixtures (tests/golden/*.npz)."""

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def _group(path):
    data = np.load(path, allow_pickle=False)
    cases = {}
    for key in data.files:
        case, name = key.rsplit("|", 1)
        cases.setdefault(case, {})[name] = data[key]
    return cases


def kernel_cases():
    """{"kernel|dtype|MxNxK|seed": {input name: array, "ref": fp32, ["triton": bits]}}"""
    return _group(GOLDEN / "reference_kernels.npz")


def routing_cases():
    return _group(GOLDEN / "routing.npz")


def parse_key(key):
    kernel, dtype, shape, seed = key.split("|")
    m, n, k = (int(v) for v in shape.split("x"))
    return kernel, dtype, (m, n, k), int(seed)

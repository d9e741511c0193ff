"""The C-ABI library loads on a CPU-only machine and exports every declared symbol."""

import ctypes
import re
from pathlib import Path

import pytest

from flashattentionanycard_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "bokt.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bokt_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_operator_entry_points():
    names = declared_symbols()
    for required in ("bokt_gemm", "bokt_rmsnorm", "bokt_moe_grouped_gemm", "bokt_moe_route",
                     "bokt_last_error", "bokt_kernel_attrs"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version_and_arch():
    lib = _native.load()
    assert lib.bokt_abi_version() == _native.ABI_VERSION
    assert lib.bokt_built_sm() == 100


def test_argument_errors_need_no_gpu():
    lib = _native.load()
    p = _native.BoktParams()
    rc = lib.bokt_gemm(None, None, None, 4, 4, 4, 7, ctypes.byref(p), None)
    assert rc == 1 and b"dtype" in lib.bokt_last_error()
    assert lib.bokt_rmsnorm(None, None, None, -1, 4, 1e-6, 1, ctypes.byref(p), None) == 1
    assert lib.bokt_moe_grouped_gemm(None, None, None, 0, None, 4, 5000, 8, 8, 1, 1,
                                     ctypes.byref(p), None) == 2
    # Empty problems are successful no-ops.
    assert lib.bokt_gemm(None, None, None, 0, 4, 4, 1, ctypes.byref(p), None) == 0
    assert lib.bokt_rmsnorm(None, None, None, 3, 0, 1e-6, 0, ctypes.byref(p), None) == 0
    assert lib.bokt_moe_route(None, 0, 0, None, None, None, None, None, None, 0, None) == 1


def test_route_workspace_size():
    lib = _native.load()
    assert lib.bokt_moe_route_workspace_bytes(32768, 64) == 8 * 64 * 4
    assert lib.bokt_moe_route_workspace_bytes(1, 3) == 1 * 3 * 4
    assert lib.bokt_moe_route_workspace_bytes(0, 3) == 3 * 4


def test_params_conversion():
    p = _native.make_params({"BLOCK_N": 128, "num_stages": 3, "GROUP_M": 4})
    assert (p.block_n, p.stages, p.group_m) == (128, 3, 4)
    with pytest.raises(ValueError):
        _native.make_params({"BLOCK_Q": 1})
    with pytest.raises(ValueError):
        _native.make_params({"BLOCK_N": 128.0})


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setenv("BOKT_LIBRARY", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="not built"):
        _native.load()
    monkeypatch.delenv("BOKT_LIBRARY")
    monkeypatch.setattr(_native, "_lib", None)
    assert _native.load() is not None


def declared_arities():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for name, params in re.findall(r"\b(bokt_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_header_arity():
    """Every ctypes binding passes exactly as many arguments as the C declaration."""
    arities = declared_arities()
    assert arities, "no declarations parsed"
    for name, n in arities.items():
        assert len(_native.SIGNATURES[name][1]) == n, (name, n, len(_native.SIGNATURES[name][1]))

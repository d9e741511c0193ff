"""Bit-exact parity of the device MoE routing front end with the oracle, and
the routed grouped GEMM end to end (route -> gather -> grouped GEMM)."""

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native
from flashattentionanycard_b200.kernels import moe_grouped_gemm
from flashattentionanycard_b200.kernels.moe_routing import MoeRouter, gather_rows
from flashattentionanycard_b200.workloads import zipf_routing
from oracle import numerics, routing
from tests.golden_cases import routing_cases
from tests.gpu_helpers import as_f32, gate

pytestmark = pytest.mark.gpu

ROUTING = routing_cases()


@pytest.fixture(autouse=True)
def clean_status(cuda_device):
    _native.device_status(reset=True)
    yield


def device_route(ids, experts, device):
    ids_d = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).to(device)
    r = MoeRouter(ids_d.numel(), experts, device, with_offsets64=True)
    r(ids_d)
    torch.cuda.synchronize()
    return r


def assert_route_equal(r, ids, experts):
    counts, offsets, perm, inv = routing.route(ids, experts)
    assert np.array_equal(r.counts.cpu().numpy(), counts)
    assert np.array_equal(r.offsets.cpu().numpy(), offsets.astype(np.int32))
    assert np.array_equal(r.offsets64.cpu().numpy(), offsets)
    assert np.array_equal(r.perm.cpu().numpy(), perm)
    assert np.array_equal(r.inv_perm.cpu().numpy(), inv)


@pytest.mark.parametrize("key", sorted(ROUTING))
def test_routing_golden(key, cuda_device):
    case = ROUTING[key]
    experts = int(key.split("|")[2])
    r = device_route(case["ids"], experts, cuda_device)
    assert np.array_equal(r.counts.cpu().numpy(), case["counts"])
    assert np.array_equal(r.offsets64.cpu().numpy(), case["offsets"])
    assert np.array_equal(r.perm.cpu().numpy(), case["perm"])
    assert_route_equal(r, case["ids"], experts)


@pytest.mark.parametrize(
    "tokens,experts,seed",
    [(16384, 64, 0), (16384, 64, 1), (3000, 8, 2), (1, 64, 0), (12289, 1000, 4)],
)
def test_routing_zipf_full_size(tokens, experts, seed, cuda_device):
    """Full benchmark size (16384 tokens, top-2, 64 experts) and ragged chunk counts."""
    ids = zipf_routing(tokens, experts, 2, 1.1, seed).numpy().reshape(-1)
    r = device_route(ids, experts, cuda_device)
    assert_route_equal(r, ids, experts)
    assert _native.device_status(reset=True)[0] == 0


def test_routing_edge_cases(cuda_device):
    for ids, experts in (
        (np.full(9000, 3, np.int32), 4),                 # one expert takes everything
        (np.arange(5000, dtype=np.int32) % 7, 7),        # round robin
        (np.zeros(0, np.int32), 5),                      # empty
        (np.array([1023] * 33 + [0] * 31, np.int32), 1024),  # maximum expert count
    ):
        if ids.size == 0:
            d = torch.zeros(0, dtype=torch.int32, device=cuda_device)
            r = MoeRouter(0, experts, cuda_device, with_offsets64=True)
            r(d)
            torch.cuda.synchronize()
            assert r.counts.sum().item() == 0 and r.offsets.cpu().tolist() == [0] * (experts + 1)
            continue
        r = device_route(ids, experts, cuda_device)
        assert_route_equal(r, ids, experts)


def test_routing_rejects_out_of_range_id_on_host_visible_status(cuda_device):
    """An id outside [0, E) sets the device status word (no trap, no fault)."""
    ids = torch.tensor([0, 1, 7, 2], dtype=torch.int32, device=cuda_device)
    r = MoeRouter(4, 4, cuda_device)
    r(ids)
    code, detail = _native.device_status(reset=True)
    assert code == 2 and detail == 2


def test_gather_rows_matches_index(cuda_device):
    src = torch.randn(300, 136, device=cuda_device).bfloat16()
    index = torch.randint(0, 600, (1000,), dtype=torch.int32, device=cuda_device)
    out = torch.empty(1000, 136, device=cuda_device, dtype=torch.bfloat16)
    gather_rows(src, index, out, divisor=2)
    torch.cuda.synchronize()
    assert torch.equal(out, src[(index // 2).long()])
    odd = torch.randn(10, 5, device=cuda_device).half()  # 10-byte rows: byte path
    out2 = torch.empty(4, 5, device=cuda_device).half()
    idx = torch.tensor([9, 0, 3, 3], dtype=torch.int32, device=cuda_device)
    gather_rows(odd, idx, out2)
    torch.cuda.synchronize()
    assert torch.equal(out2, odd[idx.long()])


def test_routed_grouped_gemm_end_to_end(cuda_device):
    """ids -> device route -> gather X in expert order -> grouped GEMM reading
    the kernel-produced int32 offsets; each assignment's output row (found
    through inv_perm) equals x[token] @ W[expert]."""
    tokens, experts, k, n = 3000, 16, 256, 512
    ids = zipf_routing(tokens, experts, 2, 1.1, 7)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(tokens, k, generator=g).bfloat16()
    w = (0.05 * torch.randn(experts, k, n, generator=g)).bfloat16()
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    r = MoeRouter(tokens * 2, experts, cuda_device)
    r(ids.to(cuda_device).reshape(-1))
    packed = torch.empty(tokens * 2, k, device=cuda_device, dtype=torch.bfloat16)
    gather_rows(xd, r.perm, packed, divisor=2)
    y = torch.full((tokens * 2, n), float("nan"), device=cuda_device, dtype=torch.bfloat16)
    moe_grouped_gemm.launch(packed, wd, r.offsets, y, {}, 148)
    torch.cuda.synchronize()
    flat = ids.reshape(-1).numpy()
    inv = r.inv_perm.cpu().numpy()
    xf, wf = as_f32(x), as_f32(w)
    ref = np.empty((tokens * 2, n), np.float32)
    for e in range(experts):
        sel = np.nonzero(flat == e)[0]
        ref[inv[sel]] = numerics.gemm_fp32(xf[sel // 2], wf[e])
    gate(y, ref, "bf16")

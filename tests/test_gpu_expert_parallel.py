"""Expert-parallel MoE on the GPU.

* ``test_virtual_ranks_on_one_gpu``: G ranks of ExpertParallelMoE on one GPU,
  the two all-to-alls done as device copies between the ranks' buffers.  Every
  device-side order (global routing, send / receive / local sorts and their
  sizes) must equal the oracle's bit for bit; outputs pass the gate (bf16 rtol
  0.02 / atol 0.15, normwise <= 1e-2) against x[token] @ W[expert] in fp32.
* ``test_nccl_two_ranks``: the real thing under torchrun with NCCL when the
  machine has at least two GPUs (skipped, with the reason, on one GPU).
"""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native
from flashattentionanycard_b200 import expert_parallel as ep
from flashattentionanycard_b200.configs.search_spaces import default_params
from flashattentionanycard_b200.workloads import zipf_routing
from oracle import numerics
from oracle import expert_parallel as oracle_ep
from tests.gpu_helpers import as_f32, gate

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


def build_ranks(world, tokens, experts, k, n, seed, device, params=None):
    ids_cpu = zipf_routing(tokens, experts, 2, 1.1, seed).reshape(-1)
    ids = ids_cpu.numpy()
    counts = np.bincount(ids, minlength=experts)
    placement = ep.plan_placement(counts, world)
    tpr = tokens // world
    plan = ep.plan_splits(ids, placement, 2, tpr)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, k, generator=g).bfloat16()
    w = (0.05 * torch.randn(experts, k, n, generator=g)).bfloat16()
    wd = w.to(device)
    ranks = []
    for r in range(world):
        lw = wd[ep.local_weight_slices(placement, r)].contiguous()
        ranks.append(ep.ExpertParallelMoE(lw, placement, plan, r, world, 2, tpr, params=params))
    return ids_cpu, ids, x, w, placement, plan, ranks


def exchange(ranks, src_attr, dst_attr, src_sizes_attr, dst_sizes_attr):
    """all_to_all emulation: chunk d of rank r's src -> chunk r of rank d's dst."""
    world = len(ranks)
    for d in range(world):
        dst = getattr(ranks[d], dst_attr)
        pos = 0
        for r in range(world):
            sizes = getattr(ranks[r], src_sizes_attr)
            start = sum(sizes[:d])
            size = sizes[d]
            assert size == getattr(ranks[d], dst_sizes_attr)[r]
            if size:
                dst[pos:pos + size].copy_(getattr(ranks[r], src_attr)[start:start + size])
            pos += size


@pytest.mark.parametrize("world", [2, 4])
def test_virtual_ranks_on_one_gpu(world, cuda_device):
    tokens, experts, k, n = 2048, 16, 256, 512
    ids_cpu, ids, x, w, placement, plan, ranks = build_ranks(world, tokens, experts, k, n, 3,
                                                             cuda_device)
    _native.device_status(reset=True)
    tpr = tokens // world
    ids_dev = ids_cpu.to(cuda_device).to(torch.int32)
    xd = x.to(cuda_device)
    for r, m in enumerate(ranks):
        m.ids_global.copy_(ids_dev)
        m.route()
        m.pack_send(xd[r * tpr:(r + 1) * tpr])
    exchange(ranks, "send_x", "recv_x", "send_sizes", "recv_sizes")
    for m in ranks:
        m.unpack_recv()
        m.compute()
        m.pack_return()
    exchange(ranks, "y_send", "y_ret", "recv_sizes", "send_sizes")
    outs = [m.unpack_return() for m in ranks]
    torch.cuda.synchronize()
    assert _native.device_status(reset=True)[0] == 0
    xf, wf = as_f32(x), as_f32(w)
    for r, m in enumerate(ranks):
        o = oracle_ep.rank_orders(ids, placement, 2, tpr, r)
        assert np.array_equal(m.route_global.perm.cpu().numpy(), o["perm"])
        assert np.array_equal(m.route_send.perm.cpu().numpy(), o["send_full"])
        assert np.array_equal(m.route_recv.perm.cpu().numpy(), o["recv_full"])
        assert np.array_equal(m.route_local.perm.cpu().numpy(), o["local_full"])
        assert np.array_equal(m.route_local.offsets.cpu().numpy()[: m.n_local + 1],
                              o["local_offsets"])
        a = np.arange(r * tpr * 2, (r + 1) * tpr * 2)
        ref = np.einsum("ak,akn->an", xf[a // 2], wf[ids[a]])
        gate(outs[r], ref, "bf16")


def test_plan_mismatch_is_reported_not_faulted(cuda_device):
    """A routing that differs from the plan's split sizes is detected on the
    device (status code 3) before any exchange; nothing faults."""
    tokens, experts, k, n = 512, 8, 64, 64
    _, ids, _, _, placement, plan, ranks = build_ranks(2, tokens, experts, k, n, 4, cuda_device)
    _native.device_status(reset=True)
    other = zipf_routing(tokens, experts, 2, 1.1, 99).reshape(-1).to(cuda_device).to(torch.int32)
    m = ranks[0]
    m.ids_global.copy_(other)
    m.route()
    code, _ = _native.device_status(reset=True)
    assert code == 3


def test_single_rank_forward_matches_one_gpu_path(cuda_device):
    """world == 1: the EP step degenerates to route + gather + grouped GEMM."""
    tokens, experts, k, n = 1024, 8, 128, 256
    ids_cpu, ids, x, w, placement, plan, ranks = build_ranks(1, tokens, experts, k, n, 6,
                                                             cuda_device)
    out = ranks[0].forward(x.to(cuda_device), ids_cpu.to(cuda_device).to(torch.int32))
    torch.cuda.synchronize()
    a = np.arange(tokens * 2)
    ref = np.einsum("ak,akn->an", as_f32(x)[a // 2], as_f32(w)[ids[a]])
    gate(out, ref, "bf16")


def test_nccl_two_ranks(cuda_device):
    """Real ranks on two GPUs: the NCCL path, the peer path with device
    barriers (eager and captured in a CUDA graph) and with NCCL barriers, a
    routing that differs from the plan; all results identical and exact."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs for a real NCCL run; the virtual-rank test covers one GPU")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29617",
           str(REPO / "tests" / "ep_nccl_check.py")]
    run = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True,
                         text=True, cwd=REPO)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
    assert "EP_NCCL_OK" in run.stdout


def build_peer_ranks(world, tokens, experts, k, n, seed, device, dtype=torch.bfloat16,
                     params=None, capacity="worst"):
    ids_cpu = zipf_routing(tokens, experts, 2, 1.1, seed).reshape(-1)
    ids = ids_cpu.numpy()
    placement = ep.plan_placement(np.bincount(ids, minlength=experts), world)
    tpr = tokens // world
    plan = ep.plan_splits(ids, placement, 2, tpr)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, k, generator=g).to(dtype)
    w = (0.05 * torch.randn(experts, k, n, generator=g)).to(dtype)
    wd = w.to(device)
    ranks = [ep.PeerExpertParallelMoE(wd[ep.local_weight_slices(placement, r)].contiguous(),
                                      placement, plan, r, world, 2, tpr, params=params,
                                      exchange=False, capacity=capacity)
             for r in range(world)]
    xpk = [m.x_packed.data_ptr() for m in ranks]
    outs = [m.out.data_ptr() for m in ranks]
    for m in ranks:
        m.set_peer_pointers(xpk, outs)
    return ids_cpu, ids, x, w, placement, ranks


@pytest.mark.parametrize("world,dtype,kernel", [(2, "bf16", "single"), (4, "bf16", "single"),
                                               (8, "bf16", "single"), (4, "fp16", "single"),
                                               (4, "bf16", "pairs"), (8, "bf16", "pairs"),
                                               (2, "fp16", "pairs")])
def test_peer_path_virtual_ranks_on_one_gpu(world, dtype, kernel, cuda_device):
    """Dispatch stores and the scatter epilogue write into other ranks' buffers
    (here: other buffers of the same GPU); the result must equal the oracle.
    ``single``: the library defaults (single-CTA grouped GEMM); ``pairs``: the
    MoE default parameters (CTA-pair grouped GEMM with half-height tails)."""
    tokens, experts, k, n = 4096, 32, 256, 512
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    params = default_params("moe_grouped_gemm") if kernel == "pairs" else None
    ids_cpu, ids, x, w, placement, ranks = build_peer_ranks(world, tokens, experts, k, n, 11,
                                                            cuda_device, tdt, params)
    _native.device_status(reset=True)
    tpr = tokens // world
    ids_dev = ids_cpu.to(cuda_device).to(torch.int32)
    xd = x.to(cuda_device)
    for r, m in enumerate(ranks):
        m.out.fill_(float("nan"))
        m.ids_global.copy_(ids_dev)
        m.layout()
    for r, m in enumerate(ranks):
        m.dispatch(xd[r * tpr:(r + 1) * tpr])
    for m in ranks:
        m.compute_and_combine()
    torch.cuda.synchronize()
    assert _native.device_status(reset=True)[0] == 0
    xf, wf = as_f32(x), as_f32(w)
    for r, m in enumerate(ranks):
        assert m.rank_rows.cpu().tolist() == [int(v) for v in placement.rank_rows]
        a = np.arange(r * tpr * 2, (r + 1) * tpr * 2)
        ref = np.einsum("ak,akn->an", xf[a // 2], wf[ids[a]])
        gate(m.out, ref, dtype)


def test_peer_path_single_rank_forward(cuda_device):
    tokens, experts, k, n = 2048, 16, 128, 256
    ids_cpu, ids, x, w, placement, ranks = build_peer_ranks(1, tokens, experts, k, n, 12,
                                                            cuda_device)
    m = ranks[0]
    for _ in range(2):
        out = m.forward(x.to(cuda_device), ids_cpu.to(cuda_device).to(torch.int32))
    torch.cuda.synchronize()
    a = np.arange(tokens * 2)
    gate(out, np.einsum("ak,akn->an", as_f32(x)[a // 2], as_f32(w)[ids[a]]), "bf16")


def run_peer_phases(ranks, ids_dev, xd, tpr):
    """One peer-path step of ranks sharing this GPU: each phase for every rank
    in turn (stream order stands in for the device barriers)."""
    for m in ranks:
        m.out.fill_(float("nan"))
        m.ids_global.copy_(ids_dev)
        m.layout()
    for r, m in enumerate(ranks):
        m.dispatch(xd[r * tpr:(r + 1) * tpr])
    for m in ranks:
        m.compute_and_combine()


@pytest.mark.parametrize("capacity", ["worst", "plan"])
def test_peer_path_routing_differs_from_plan(capacity, cuda_device):
    """The placement comes from one routing, the step sees another that piles
    every token on experts 0 and 1.  With worst-case capacity (the default) the
    result is still exact; with plan-sized buffers the overflow is reported
    (status 4) instead of silently dropping rows, and forward-style checking
    raises."""
    world, tokens, experts, k, n = 4, 2048, 16, 128, 256
    ids_cpu, ids, x, w, placement, ranks = build_peer_ranks(world, tokens, experts, k, n, 21,
                                                            cuda_device, capacity=capacity)
    step_ids = torch.tensor([[0, 1]] * tokens, dtype=torch.int32).reshape(-1)
    tpr = tokens // world
    _native.device_status(reset=True)
    run_peer_phases(ranks, step_ids.to(cuda_device), x.to(cuda_device), tpr)
    torch.cuda.synchronize()
    if capacity == "plan":
        with pytest.raises(RuntimeError, match="too small"):
            ep.check_device_status("step")
        return
    ep.check_device_status("step")
    xf, wf, sid = as_f32(x), as_f32(w), step_ids.numpy()
    for r, m in enumerate(ranks):
        a = np.arange(r * tpr * 2, (r + 1) * tpr * 2)
        gate(m.out, np.einsum("ak,akn->an", xf[a // 2], wf[sid[a]]), "bf16")


def _ptrs(tensors, device):
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device=device)


def test_device_barrier_success_and_timeout(cuda_device):
    """bokt_ep_barrier as rank 0 of 2, both flag arrays in this GPU's memory.
    First call: the peer never signals -> the wait gives up after 50 ms,
    records status 1 with detail 4001 (rank 1) and returns; this rank's signal
    reached both arrays.  Second call with the peer's signal already in place:
    passes with no status.  A GEMM right after runs normally."""
    lib = _native.load()
    stream = _native.current_stream(cuda_device)
    mine = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    peer = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ptrs = _ptrs([mine, peer], cuda_device)
    _native.device_status(reset=True)
    _native.check(lib.bokt_ep_barrier(ptrs.data_ptr(), epoch.data_ptr(), 2, 0, 50_000_000,
                                      stream), "barrier")
    assert _native.device_status(reset=True) == (1, 4001)
    assert epoch.item() == 1 and mine[0].item() == 1 and peer[0].item() == 1
    mine[1] = 2  # rank 1 has already reached barrier 2
    _native.check(lib.bokt_ep_barrier(ptrs.data_ptr(), epoch.data_ptr(), 2, 0, 50_000_000,
                                      stream), "barrier")
    assert _native.device_status(reset=True) == (0, 0)
    assert epoch.item() == 2 and peer[0].item() == 2
    a = torch.randn(256, 384, device=cuda_device).bfloat16()
    b = torch.randn(384, 512, device=cuda_device).bfloat16()
    from flashattentionanycard_b200.kernels import gemm
    out = torch.empty(256, 512, device=cuda_device, dtype=torch.bfloat16)
    gemm.launch(a, b, out, {})
    torch.cuda.synchronize()
    gate(out, as_f32(a.cpu()) @ as_f32(b.cpu()), "bf16")


def test_put_copies_into_every_rank(cuda_device):
    lib = _native.load()
    world, chunk = 3, 96
    src = torch.arange(chunk, dtype=torch.int32, device=cuda_device) + 7
    dsts = [torch.full((world * chunk,), -1, dtype=torch.int32, device=cuda_device)
            for _ in range(world)]
    _native.check(lib.bokt_ep_put(src.data_ptr(), chunk * 4, _ptrs(dsts, cuda_device).data_ptr(),
                                  1 * chunk * 4, world, _native.current_stream(cuda_device)),
                  "put")
    torch.cuda.synchronize()
    for d in dsts:
        assert torch.equal(d[chunk:2 * chunk], src)
        assert int(d[:chunk].max()) == -1 and int(d[2 * chunk:].max()) == -1

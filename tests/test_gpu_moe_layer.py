"""Routing front end and combine on the GPU: top-k softmax gate (expert ids
bit-exact, gates within 1e-5 relative), gate-weighted combine, and a whole MoE
layer (logits -> gate -> route -> gather -> grouped GEMM -> combine) against
the oracle with the reference gate (bf16 rtol 0.02 / atol 0.15, normwise <= 1e-2)."""

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native
from flashattentionanycard_b200.kernels import moe_grouped_gemm
from flashattentionanycard_b200.kernels.moe_routing import MoeRouter, combine, gather_rows, topk_gate
from oracle import numerics, routing
from tests.gpu_helpers import as_f32, gate

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def clean_status(cuda_device):
    _native.device_status(reset=True)
    yield
    assert _native.device_status(reset=True)[0] == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(16384, 64, 2), (1000, 8, 1), (77, 1000, 8), (5, 3, 3)])
@pytest.mark.parametrize("renorm", [True, False])
def test_topk_gate(shape, dtype, renorm, cuda_device):
    t, e, k = shape
    g = torch.Generator().manual_seed(t + e)
    logits = (2 * torch.randn(t, e, generator=g)).to(dtype)
    if t > 3:
        logits[3, 0] = logits[3, e - 1] = logits[3].max() + 1  # a tie at the top
    ids = torch.full((t, k), -1, dtype=torch.int32, device=cuda_device)
    gates = torch.full((t, k), float("nan"), dtype=torch.float32, device=cuda_device)
    topk_gate(logits.to(cuda_device), k, ids, gates, renorm)
    torch.cuda.synchronize()
    want_ids, want_gates = routing.topk_gate(logits.float().numpy(), k, renorm)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    np.testing.assert_allclose(gates.cpu().numpy(), want_gates, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("with_rows", [False, True])
def test_combine(with_rows, cuda_device):
    t, k, n = 3000, 2, 520
    g = torch.Generator().manual_seed(5)
    y = torch.randn(t * k, n, generator=g).bfloat16()
    gates = torch.rand(t, k, generator=g)
    rows = torch.randperm(t * k, generator=g).to(torch.int32) if with_rows else None
    out = torch.full((t, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    combine(y.to(cuda_device), gates.to(cuda_device), out,
            rows.to(cuda_device) if with_rows else None)
    torch.cuda.synchronize()
    ref = routing.combine(as_f32(y), gates.numpy(), rows.numpy() if with_rows else None)
    gate(out, ref, "bf16")


def test_moe_layer_end_to_end(cuda_device):
    tokens, experts, k_top, hidden, n = 4096, 16, 2, 512, 1024
    g = torch.Generator().manual_seed(9)
    x = torch.randn(tokens, hidden, generator=g).bfloat16()
    logits = torch.randn(tokens, experts, generator=g)
    w = (0.05 * torch.randn(experts, hidden, n, generator=g)).bfloat16()
    dev = cuda_device
    ids = torch.empty(tokens, k_top, dtype=torch.int32, device=dev)
    gates = torch.empty(tokens, k_top, dtype=torch.float32, device=dev)
    topk_gate(logits.to(dev), k_top, ids, gates)
    r = MoeRouter(tokens * k_top, experts, dev)
    r(ids.reshape(-1))
    xd = x.to(dev)
    packed = torch.empty(tokens * k_top, hidden, dtype=torch.bfloat16, device=dev)
    gather_rows(xd, r.perm, packed, divisor=k_top)
    y = torch.empty(tokens * k_top, n, dtype=torch.bfloat16, device=dev)
    moe_grouped_gemm.launch(packed, w.to(dev), r.offsets, y, {}, 148)
    out = torch.full((tokens, n), float("nan"), dtype=torch.bfloat16, device=dev)
    combine(y, gates, out, r.inv_perm)
    torch.cuda.synchronize()
    want_ids, want_gates = routing.topk_gate(logits.numpy(), k_top)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    xf, wf = as_f32(x), as_f32(w)
    per = np.einsum("tk,tkn->tkn", np.ones((tokens, k_top), np.float32),
                    np.stack([xf @ wf[e] for e in range(experts)], 1)[np.arange(tokens)[:, None],
                                                                      want_ids])
    ref = np.einsum("tk,tkn->tn", want_gates, per)
    gate(out, ref, "bf16")


@pytest.mark.parametrize("world", [1, 2, 4])
def test_moe_layer_expert_parallel_fused_combine(world, cuda_device):
    """The MoE layer through the expert-parallel peer path with the combine
    fused into the step's last barrier (bokt_ep_barrier_combine): logits ->
    gate -> per-rank dispatch -> grouped GEMM with peer-store scatter ->
    fused combine.  Ranks share this GPU (phases in stream order).  Each rank's
    token-order output is bit-identical to the separate combine kernel run on
    the same slot rows, and passes the gate against the oracle layer."""
    from flashattentionanycard_b200 import expert_parallel as ep
    from flashattentionanycard_b200.configs.search_spaces import default_params

    tokens, experts, k_top, hidden, n = 4096, 16, 2, 512, 1024
    g = torch.Generator().manual_seed(9)
    x = torch.randn(tokens, hidden, generator=g).bfloat16()
    logits = torch.randn(tokens, experts, generator=g)
    w = (0.05 * torch.randn(experts, hidden, n, generator=g)).bfloat16()
    dev = cuda_device
    ids = torch.empty(tokens, k_top, dtype=torch.int32, device=dev)
    gates = torch.empty(tokens, k_top, dtype=torch.float32, device=dev)
    topk_gate(logits.to(dev), k_top, ids, gates)
    flat = ids.reshape(-1).cpu().numpy()
    placement = ep.plan_placement(np.bincount(flat, minlength=experts), world)
    tpr = tokens // world
    plan = ep.plan_splits(flat, placement, k_top, tpr)
    wd, xd = w.to(dev), x.to(dev)
    params = default_params("moe_grouped_gemm")
    ranks = [ep.PeerExpertParallelMoE(wd[ep.local_weight_slices(placement, r)].contiguous(),
                                      placement, plan, r, world, k_top, tpr, params=params,
                                      exchange=False) for r in range(world)]
    for m in ranks:
        m.set_peer_pointers([q.x_packed.data_ptr() for q in ranks],
                            [q.out.data_ptr() for q in ranks])
        m.ids_global.copy_(ids.reshape(-1))
        m.final.fill_(float("nan"))
        m.layout()
    for r, m in enumerate(ranks):
        m.dispatch(xd[r * tpr:(r + 1) * tpr])
    for m in ranks:
        m.compute_and_combine()
    finals = [m.barrier_combine(gates[r * tpr:(r + 1) * tpr]).clone()
              for r, m in enumerate(ranks)]
    torch.cuda.synchronize()
    want_ids, want_gates = routing.topk_gate(logits.numpy(), k_top)
    xf, wf = as_f32(x), as_f32(w)
    per = np.stack([xf @ wf[e] for e in range(experts)], 1)[np.arange(tokens)[:, None], want_ids]
    ref = np.einsum("tk,tkn->tn", want_gates, per)
    for r, m in enumerate(ranks):
        separate = torch.empty(tpr, n, dtype=torch.bfloat16, device=dev)
        combine(m.out, gates[r * tpr:(r + 1) * tpr], separate)
        torch.cuda.synchronize()
        assert torch.equal(finals[r], separate), "fused combine differs from the combine kernel"
        gate(finals[r], ref[r * tpr:(r + 1) * tpr], "bf16")

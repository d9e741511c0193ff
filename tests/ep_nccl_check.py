"""torchrun worker for tests/test_gpu_expert_parallel.py::test_nccl_two_ranks.

Each rank owns a block of tokens, holds only its virtual experts' weights, and
runs ExpertParallelMoE.forward with NCCL all-gather / all-to-all, then the
peer-memory path with device barriers (eager, and captured in a CUDA graph)
and with NCCL barriers, and a step whose routing differs from the plan.  Rank
outputs are checked against x[token] @ W[expert] (fp32) with the reference
gate and must be bit-identical across the paths.
"""

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from flashattentionanycard_b200 import _native  # noqa: E402
from flashattentionanycard_b200 import expert_parallel as ep  # noqa: E402
from flashattentionanycard_b200.workloads import zipf_routing  # noqa: E402
from oracle import numerics  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=device)
    tokens, experts, k, n = 4096, 16, 256, 512
    tpr = tokens // world
    ids_all = zipf_routing(tokens, experts, 2, 1.1, 8).reshape(-1)
    g = torch.Generator().manual_seed(8)
    x = torch.randn(tokens, k, generator=g).bfloat16()
    w = (0.05 * torch.randn(experts, k, n, generator=g)).bfloat16()
    ids = ids_all.numpy()
    placement = ep.plan_placement(np.bincount(ids, minlength=experts), world)
    plan = ep.plan_splits(ids, placement, 2, tpr)
    lw = w[ep.local_weight_slices(placement, rank)].contiguous().to(device)
    m = ep.ExpertParallelMoE(lw, placement, plan, rank, world, 2, tpr)
    ids_local = ids_all[rank * tpr * 2:(rank + 1) * tpr * 2].to(torch.int32).to(device)
    out = None
    for _ in range(2):  # twice: buffers are reused across steps
        out = m.forward(x[rank * tpr:(rank + 1) * tpr].to(device), ids_local)
    torch.cuda.synchronize()
    code, detail = _native.device_status(reset=True)
    a = np.arange(rank * tpr * 2, (rank + 1) * tpr * 2)
    ref = np.einsum("ak,akn->an", x.float().numpy()[a // 2], w.float().numpy()[ids[a]])
    stats = numerics.check_output(out.float().cpu().numpy(), ref, "bf16")
    xl = x[rank * tpr:(rank + 1) * tpr].to(device)
    results = {}
    # Peer-memory path (CUDA IPC + NVLink stores), device barriers and NCCL barriers.
    for sync in ("device", "nccl"):
        pm = ep.PeerExpertParallelMoE(lw, placement, plan, rank, world, 2, tpr, sync=sync)
        for _ in range(2):
            pout = pm.forward(xl, ids_local, check=True)
        torch.cuda.synchronize()
        results[sync] = (pout.clone(), pm)
    # The device-barrier step captured in a CUDA graph (no host collective inside).
    pm = results["device"][1]
    stream = torch.cuda.Stream(device)
    graph = torch.cuda.CUDAGraph()
    dist.barrier()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(3):
            pm.forward(xl, ids_local)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    gout = pm.out.clone()
    del graph
    ep.check_device_status("graph replay")
    # A routing the plan was not made for (all tokens on experts 0 and 1).
    other = torch.tensor([[0, 1]] * tpr, dtype=torch.int32, device=device).reshape(-1)
    oout = pm.forward(xl, other, check=True).clone()
    torch.cuda.synchronize()
    code2, _ = _native.device_status(reset=True)
    pstats = numerics.check_output(results["device"][0].float().cpu().numpy(), ref, "bf16")
    oa = np.arange(rank * tpr * 2, (rank + 1) * tpr * 2)
    oids = np.tile([0, 1], tpr)
    oref = np.einsum("ak,akn->an", x.float().numpy()[oa // 2], w.float().numpy()[oids])
    ostats = numerics.check_output(oout.float().cpu().numpy(), oref, "bf16")
    same = bool(torch.equal(results["device"][0], out) and torch.equal(results["nccl"][0], out)
                and torch.equal(gout, out))
    dist.barrier()
    for _, m in results.values():
        m.close()
    code = code or code2
    ok = torch.tensor([1 if code == 0 and same else 0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and ok.item() == 1:
        print(f"EP_NCCL_OK rel={stats['normwise_rel_error']:.2e} "
              f"peer rel={pstats['normwise_rel_error']:.2e} other-routing "
              f"rel={ostats['normwise_rel_error']:.2e} identical={same}")
    return 0 if ok.item() == 1 else 1


if __name__ == "__main__":
    sys.exit(main())

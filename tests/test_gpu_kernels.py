"""GPU parity of the sm_100a kernels against the CPU oracle.

Tolerance (every numeric test): the reference's FP32 gate, fp16 rtol 0.01 /
atol 0.02 and bf16 rtol 0.02 / atol 0.15 (reference worker.py:111), plus a
normwise relative error ||out - ref|| / ||ref|| <= 1e-2.  Outputs are
NaN-prefilled so an unwritten element fails (reference worker.py:187).
"""

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native
from flashattentionanycard_b200.configs.search_spaces import Workload, grid_configs, search_space
from flashattentionanycard_b200.kernels import gemm, moe_grouped_gemm, rmsnorm
from flashattentionanycard_b200.tuner import worker
from flashattentionanycard_b200.tuner.hardware import Hardware, prune_reason
from oracle import numerics
from tests.golden_cases import kernel_cases, parse_key
from tests.gpu_helpers import as_f32, from_bits, gate, nan_like

pytestmark = pytest.mark.gpu

CASES = kernel_cases()


@pytest.fixture(autouse=True)
def clean_status(cuda_device):
    _native.device_status(reset=True)
    yield
    code, detail = _native.device_status(reset=True)
    assert code == 0, f"device status {code} (detail {detail})"


def run_case(kernel, dtype, case, params, device, sm_count):
    if kernel == "gemm":
        a, b = from_bits(case["a"], dtype, device), from_bits(case["b"], dtype, device)
        out = nan_like((a.shape[0], b.shape[1]), dtype, device)
        gemm.launch(a, b, out, params)
        ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    elif kernel == "rmsnorm":
        x, w = from_bits(case["x"], dtype, device), from_bits(case["weight"], dtype, device)
        out = nan_like(tuple(x.shape), dtype, device)
        rmsnorm.launch(x, w, out, params, 1e-6)
        ref = numerics.rmsnorm_fp32(as_f32(x), as_f32(w), 1e-6)
    else:
        x, w = from_bits(case["x"], dtype, device), from_bits(case["weight"], dtype, device)
        starts = case["starts"]
        offsets = torch.tensor(starts, dtype=torch.int64, device=device)
        out = nan_like((x.shape[0], w.shape[2]), dtype, device)
        moe_grouped_gemm.launch(x, w, offsets, out, params, sm_count)
        ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    torch.cuda.synchronize()
    return out, ref


@pytest.mark.parametrize("key", sorted(CASES))
def test_golden_cases_all_smoke_configs(key, cuda_device):
    """Every golden input (drawn as the reference draws) x every smoke config."""
    kernel, dtype, _, _ = parse_key(key)
    sm = Hardware.detect(cuda_device.index).sm_count
    for params in grid_configs(search_space(kernel, "smoke")):
        out, ref = run_case(kernel, dtype, CASES[key], params, cuda_device, sm)
        gate(out, ref, dtype)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("kernel", ["gemm", "rmsnorm", "moe_grouped_gemm"])
@pytest.mark.parametrize("shape", [(64, 128, 64), (37, 77, 93), (1, 1, 1)])
def test_gpu_outputs(kernel, dtype, shape, cuda_device):
    """The reference's own GPU test (tests/test_correctness.py:550-571) through
    this worker's prepare/check_output."""
    hardware = Hardware.detect(cuda_device.index)
    m, n, k = shape
    w = Workload(kernel, m, n, k, dtype, (0, 1, 33, 0, 9))
    for p in grid_configs(search_space(kernel, "smoke")):
        for seed in (0, 17):
            call, out, reference = worker.prepare(w, cuda_device, seed, hardware.sm_count)
            out.fill_(float("nan"))
            call(p)
            torch.cuda.synchronize(cuda_device)
            worker.check_output(out, reference, dtype)


TC_SHAPES = [(1, 8, 8), (128, 256, 64), (129, 136, 72), (300, 520, 1000), (257, 264, 4104),
             (1000, 64, 128)]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", TC_SHAPES)
def test_tcgen05_gemm_edges_every_legal_config(shape, dtype, cuda_device):
    """tcgen05 path (K, N multiples of 8): ragged M/N/K tails under every legal
    (BLOCK_N, stages, GROUP_M) configuration of the full space."""
    m, n, k = shape
    g = torch.Generator().manual_seed(m * 7 + n)
    a = torch.randn(m, k, generator=g).to(worker_dtype(dtype))
    b = torch.randn(k, n, generator=g).to(worker_dtype(dtype))
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    a, b = a.to(cuda_device), b.to(cuda_device)
    hw = Hardware.detect(cuda_device.index)
    seen = 0
    for p in grid_configs(search_space("gemm")):
        if prune_reason(hw, "gemm", p) or (p["GROUP_M"] not in (1, 8)):
            continue
        out = nan_like((m, n), dtype, cuda_device)
        compiled = gemm.launch(a, b, out, p)
        assert compiled.path == "tcgen05"
        torch.cuda.synchronize()
        gate(out, ref, dtype)
        seen += 1
    assert seen >= 10


def worker_dtype(dtype):
    return {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]


@pytest.mark.parametrize("counts", [(0, 1, 33, 0, 9), (0, 0, 0, 300), (128, 0, 129, 1, 255),
                                    (0, 16, 64, 256, 1024, 32, 8, 128)])
@pytest.mark.parametrize("offset_dtype", [torch.int32, torch.int64])
def test_tcgen05_grouped_gemm_ragged_experts(counts, offset_dtype, cuda_device):
    n, k = 264, 136
    g = torch.Generator().manual_seed(len(counts))
    x = torch.randn(sum(counts), k, generator=g).bfloat16()
    w = (0.5 * torch.randn(len(counts), k, n, generator=g)).bfloat16()
    starts = [0]
    for c in counts:
        starts.append(starts[-1] + c)
    ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    offsets = torch.tensor(starts, dtype=offset_dtype, device=cuda_device)
    hw = Hardware.detect(cuda_device.index)
    for p in grid_configs(search_space("moe_grouped_gemm")):
        if prune_reason(hw, "moe_grouped_gemm", p) or p["num_stages"] not in (2, 4):
            continue
        out = nan_like((x.shape[0], n), "bf16", cuda_device)
        compiled = moe_grouped_gemm.launch(xd, wd, offsets, out, p, hw.sm_count)
        assert compiled.path == "tcgen05"
        torch.cuda.synchronize()
        gate(out, ref, "bf16")


@pytest.mark.parametrize("experts", [191, 193, 300, 1000])
def test_grouped_gemm_balanced_raster_many_experts(experts, cuda_device):
    """RASTER 2 (low-reuse experts interleaved) computes the same tiles as
    RASTER 1, bit for bit; experts not a multiple of 32 exercise uneven runs
    per lane of the warp that builds the schedule."""
    n, k = 136, 72
    rng = np.random.default_rng(experts)
    counts = rng.integers(0, 400, size=experts)
    counts[rng.integers(0, experts, size=experts // 5)] = 0
    starts = np.concatenate([[0], np.cumsum(counts)]).tolist()
    g = torch.Generator().manual_seed(experts)
    x = torch.randn(starts[-1], k, generator=g).bfloat16()
    w = (0.5 * torch.randn(experts, k, n, generator=g)).bfloat16()
    ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    offsets = torch.tensor(starts, dtype=torch.int32, device=cuda_device)
    outs = []
    for raster in (1, 2):
        out = nan_like((x.shape[0], n), "bf16", cuda_device)
        moe_grouped_gemm.launch(xd, wd, offsets, out,
                                {"BLOCK_N": 128, "num_stages": 4, "RASTER": raster}, 148)
        torch.cuda.synchronize()
        gate(out, ref, "bf16")
        outs.append(out)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("params", [{"BLOCK_N": 256, "num_stages": 6, "CTA_GROUP": 2},
                                    {"BLOCK_N": 128, "num_stages": 8, "CTA_GROUP": 2},
                                    {"BLOCK_N": 256, "num_stages": 4, "CTA_GROUP": 2,
                                     "RASTER": 2}])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_grouped_gemm_pair_tiles_cover_every_row(params, dtype, cuda_device):
    """CTA_GROUP 2: 256-row pair tiles per expert, a last block of <= 128 rows
    as a half-height pair tile (M = 128, 64 rows per CTA).  Expert sizes around
    every multiple of 128 and 256; every row of the NaN-prefilled output is
    written exactly as the oracle says, rows before offsets[0] / after
    offsets[E] stay NaN, and the single-CTA kernel agrees."""
    n, k = 392, 200
    sizes = [0, 1, 127, 128, 129, 255, 256, 257, 383, 384, 385, 511, 512, 513, 700, 1000]
    rng = np.random.default_rng(1)
    counts = sizes + rng.integers(0, 600, size=20).tolist()
    lead, trail = 3, 5
    starts = [lead]
    for c in counts:
        starts.append(starts[-1] + c)
    rows = starts[-1] + trail
    g = torch.Generator().manual_seed(7)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    x = torch.randn(rows, k, generator=g).to(tdt)
    w = (0.5 * torch.randn(len(counts), k, n, generator=g)).to(tdt)
    ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    out = nan_like((rows, n), dtype, cuda_device)
    offsets = torch.tensor(starts, dtype=torch.int64, device=cuda_device)
    compiled = moe_grouped_gemm.launch(x.to(cuda_device), w.to(cuda_device), offsets, out,
                                       params, 148)
    torch.cuda.synchronize()
    assert compiled.path == "tcgen05" and compiled.n_spills == 0
    got = out.float().cpu().numpy()
    assert np.isnan(got[:lead]).all() and np.isnan(got[rows - trail:]).all()
    gate(out[lead:rows - trail], ref[lead:rows - trail], dtype)
    single = nan_like((rows, n), dtype, cuda_device)
    moe_grouped_gemm.launch(x.to(cuda_device), w.to(cuda_device), offsets, single,
                            dict(params, CTA_GROUP=1, num_stages=4), 148)
    torch.cuda.synchronize()
    diff = (single[lead:rows - trail].float() - out[lead:rows - trail].float()).abs().max().item()
    assert diff <= 0.05 * float(np.nanmax(np.abs(ref)))


def test_grouped_gemm_leaves_rows_outside_experts(cuda_device):
    """Rows before offsets[0] and after offsets[E] are not written (reference
    kernel writes only [start, start + count) per expert)."""
    n, k = 64, 64
    x = torch.randn(40, k).bfloat16()
    w = torch.randn(2, k, n).bfloat16()
    starts = [5, 20, 31]
    ref = numerics.grouped_gemm_fp32(as_f32(x), as_f32(w), starts)
    out = nan_like((40, n), "bf16", cuda_device)
    offsets = torch.tensor(starts, dtype=torch.int32, device=cuda_device)
    moe_grouped_gemm.launch(x.to(cuda_device), w.to(cuda_device), offsets, out,
                            {"BLOCK_N": 64, "num_stages": 2}, 148)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isnan(got[:5]).all() and np.isnan(got[31:]).all()
    gate(out[5:31], ref[5:31], "bf16")


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 8), (3, 4096), (37, 77), (513, 520), (64, 16384),
                                   (7, 65536), (2, 5)])
def test_rmsnorm_every_config(shape, dtype, cuda_device):
    m, n = shape
    g = torch.Generator().manual_seed(n)
    x = torch.randn(m, n, generator=g).to(worker_dtype(dtype))
    w = (1 + 0.1 * torch.randn(n, generator=g)).to(worker_dtype(dtype))
    ref = numerics.rmsnorm_fp32(as_f32(x), as_f32(w), 1e-6)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    hw = Hardware.detect(cuda_device.index)
    for p in grid_configs(search_space("rmsnorm")):
        if prune_reason(hw, "rmsnorm", p, n):
            continue
        out = nan_like((m, n), dtype, cuda_device)
        rmsnorm.launch(xd, wd, out, p, 1e-6)
        torch.cuda.synchronize()
        gate(out, ref, dtype)


def test_unaligned_pointer_takes_edge_path(cuda_device):
    """A view starting 2 bytes into a buffer is not 16-byte aligned: the
    library must not hand it to TMA."""
    base = torch.randn(1, 64 * 64 + 1).bfloat16()
    a_cpu = base[0, 1:].reshape(64, 64)
    b_cpu = torch.randn(64, 64).bfloat16()
    ref = numerics.gemm_fp32(as_f32(a_cpu), as_f32(b_cpu))
    dev = base.to(cuda_device)
    a = dev[0, 1:].view(64, 64)
    assert a.data_ptr() % 16 != 0
    out = nan_like((64, 64), "bf16", cuda_device)
    gemm.launch(a, b_cpu.to(cuda_device), out, {})
    torch.cuda.synchronize()
    gate(out, ref, "bf16")


def test_launch_errors_raise(cuda_device):
    a = torch.randn(64, 64, device=cuda_device).bfloat16()
    out = torch.empty(64, 64, device=cuda_device).bfloat16()
    with pytest.raises(RuntimeError, match="block_n"):
        gemm.launch(a, a, out, {"BLOCK_N": 96})
    with pytest.raises(RuntimeError, match="shared memory"):
        gemm.launch(a, a, out, {"BLOCK_N": 256, "num_stages": 8})
    with pytest.raises(ValueError):
        gemm.launch(a, a.half(), out, {})
    with pytest.raises(RuntimeError, match="num_warps"):
        rmsnorm.launch(a, a[0].contiguous(), out, {"num_warps": 3})


def test_compiled_metadata_fields(cuda_device):
    a = torch.randn(256, 256, device=cuda_device).bfloat16()
    out = torch.empty_like(a)
    compiled = gemm.launch(a, a, out, {"BLOCK_N": 128, "num_stages": 4})
    hw = Hardware.detect(cuda_device.index)
    assert 0 < compiled.metadata.shared <= hw.shared_memory_per_block
    assert compiled.n_regs > 0 and compiled.n_spills == 0 and compiled.threads == 192
    c2 = rmsnorm.launch(a, a[0].contiguous(), out, {"ROWS_PER_CTA": 1, "num_warps": 4})
    assert c2.path == "vector" and c2.n_spills == 0


@pytest.mark.parametrize("kernel", ["gemm", "rmsnorm", "moe_grouped_gemm"])
def test_launch_is_graph_capturable(kernel, cuda_device):
    """No sync, allocation or host read-back inside launch: a CUDA graph of the
    call replays to the same result (reference worker.py:148-151)."""
    hw = Hardware.detect(cuda_device.index)
    w = Workload(kernel, 256, 512, 384, "bf16", (100, 0, 300, 12))
    call, out, ref = worker.prepare(w, cuda_device, 3, hw.sm_count)
    p = next(grid_configs(search_space(kernel, "smoke")))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call(p)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    out.fill_(float("nan"))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        call(p)
    graph.replay()
    torch.cuda.synchronize()
    worker.check_output(out, ref, "bf16")


def test_cuda_measurement(cuda_device):
    x = torch.ones(1024, device=cuda_device)
    result = worker.measure(lambda: x.add_(1), worker.Measurement(2, 3, 2, 1))
    assert len(result["samples_ms"]) == 3
    assert result["latency_ms"] > 0


@pytest.mark.parametrize("kernel", ["gemm", "rmsnorm", "moe_grouped_gemm"])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_worker_evaluate_and_confirmation(kernel, dtype, cuda_device):
    """The full worker path: validation seeds, smem check, CUDA-graph timing,
    and the paired candidate/torch confirmation (reference test_correctness.py:586-614)."""
    from dataclasses import asdict

    workload = Workload(kernel, 37, 77, 93, dtype, (0, 1, 33, 0, 9))
    spec = {
        "device": cuda_device.index,
        "workload": asdict(workload),
        "params": next(grid_configs(search_space(kernel, "smoke"))),
        "measurement": asdict(worker.Measurement(2, 3, 2, 2)),
    }
    result = worker.evaluate(spec)
    assert result["implementation"] == worker.CANDIDATE and len(result["validation"]) == 2
    order = ["candidate", "torch"] if dtype == "fp16" else ["torch", "candidate"]
    pair = worker.evaluate_confirmation(dict(spec, order=order))
    assert pair["candidate"]["implementation"] == worker.CANDIDATE
    assert pair["torch"]["implementation"] == worker.BASELINES[kernel]


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(128, 256, 64), (256, 256, 64), (300, 520, 1000),
                                   (257, 264, 4104), (1, 8, 8), (1000, 136, 200)])
def test_cta_pair_gemm_edges(shape, dtype, cuda_device):
    """tcgen05 cta_group::2 (CTA pairs, 256-row tiles): ragged M/N/K tails,
    rows owned only by the second CTA of a pair, every stage depth."""
    m, n, k = shape
    g = torch.Generator().manual_seed(m * 13 + n)
    a = torch.randn(m, k, generator=g).to(worker_dtype(dtype))
    b = torch.randn(k, n, generator=g).to(worker_dtype(dtype))
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    a, b = a.to(cuda_device), b.to(cuda_device)
    for bn, stages in ((256, 6), (256, 3), (128, 8), (128, 4)):
        for group_m in (1, 8):
            out = nan_like((m, n), dtype, cuda_device)
            gemm.launch(a, b, out, {"BLOCK_N": bn, "num_stages": stages, "GROUP_M": group_m,
                                    "CTA_GROUP": 2})
            torch.cuda.synchronize()
            gate(out, ref, dtype)


def test_cta_pair_gemm_2048(cuda_device):
    from flashattentionanycard_b200 import workloads

    a, b = workloads.gemm_inputs(2048, 2048, 2048, "bf16", seed=1)
    ref = numerics.gemm_fp32(as_f32(a), as_f32(b))
    out = nan_like((2048, 2048), "bf16", cuda_device)
    gemm.launch(a.to(cuda_device), b.to(cuda_device), out, {"CTA_GROUP": 2})
    torch.cuda.synchronize()
    gate(out, ref, "bf16")


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 8), (3, 4096), (148, 1024), (1000, 4096), (4096, 4096),
                                   (10, 14336), (5000, 520)])
def test_rmsnorm_ring_kernel(shape, dtype, cuda_device):
    """Persistent TMA-staged RMSNorm (num_stages >= 2): fewer rows than CTAs,
    rows per CTA not a multiple of the consumer warps, wide rows."""
    m, n = shape
    g = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, n, generator=g).to(worker_dtype(dtype))
    w = (1 + 0.1 * torch.randn(n, generator=g)).to(worker_dtype(dtype))
    ref = numerics.rmsnorm_fp32(as_f32(x), as_f32(w), 1e-6)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    for warps, stages in ((8, 16), (4, 8), (1, 4), (16, 16), (2, 2)):
        p = {"ROWS_PER_CTA": 1, "num_warps": warps, "num_stages": stages}
        if n * 2 * (stages + 1) > 200 * 1024 or stages < 4:
            continue
        out = nan_like((m, n), dtype, cuda_device)
        compiled = rmsnorm.launch(xd, wd, out, p, 1e-6)
        assert compiled.path == "ring"
        torch.cuda.synchronize()
        gate(out, ref, dtype)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 8), (3, 4096), (148, 1024), (4096, 4096), (5000, 520),
                                   (20000, 2048), (7, 8192)])
def test_rmsnorm_pipelined_kernel(shape, dtype, cuda_device):
    """Persistent software-pipelined RMSNorm (num_stages 2): fewer rows than
    CTAs, several rows per CTA, next-row loads past the last row."""
    m, n = shape
    g = torch.Generator().manual_seed(3 * m + n)
    x = torch.randn(m, n, generator=g).to(worker_dtype(dtype))
    w = (1 + 0.1 * torch.randn(n, generator=g)).to(worker_dtype(dtype))
    ref = numerics.rmsnorm_fp32(as_f32(x), as_f32(w), 1e-6)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    for warps in (1, 2, 4, 8):
        out = nan_like((m, n), dtype, cuda_device)
        compiled = rmsnorm.launch(xd, wd, out, {"ROWS_PER_CTA": 1, "num_warps": warps,
                                               "num_stages": 2}, 1e-6)
        per_thread = -(-(n // 8) // (warps * 32))
        assert compiled.path == ("pipelined" if per_thread <= 8 else
                                 "vector" if per_thread <= 16 else "scalar")
        torch.cuda.synchronize()
        gate(out, ref, dtype)

"""B200 (sm_100) detection, NVLink topology, and launch-legality checks.

Mirrors the reference's ``bo_kernel_tuner/tuner/hardware.py`` (``Hardware``
:6-42, ``resource_estimate`` :45-55, ``prune_reason`` :58-74).  Differences:

* ``Hardware.detect`` requires an sm_100 device (the kernels are built for
  sm_100a only) and records the NVLink peer topology.
* ``resource_estimate`` is exact for the tcgen05 kernels: it is the formula the
  C library uses for the dynamic shared memory of the TMA ring, plus the TMEM
  columns (two accumulators of BLOCK_N fp32 columns).
* A shared-memory overflow is a hard legality failure here (the estimate is
  the real allocation), while ``heuristic_smem`` keeps its reference meaning:
  an optional, stricter pre-filter against the per-block limit.
"""

import re
import subprocess
from dataclasses import asdict, dataclass, field

GEMM_BM, GEMM_BK = 128, 64
GEMM_WARPS = 6
TMEM_COLUMNS = 512
SPLIT_K_MAX = 128  # slices per tile the library accepts (kSplitKMax)
EPILOGUE_BYTES = 4 * (32 * 128 + 32 * 8)  # staging + row pointers of the 4 epilogue warps


@dataclass(frozen=True)
class Hardware:
    name: str
    capability: tuple[int, int]
    sm_count: int
    total_memory: int
    shared_memory_per_block: int
    max_threads_per_block: int = 1024
    warp_size: int = 32
    uuid: str = "unknown"
    device: int = 0
    nvlink: dict = field(default_factory=dict, compare=False)

    def to_dict(self):
        data = asdict(self)
        data["capability"] = list(self.capability)
        return data

    @classmethod
    def detect(cls, device=0):
        import torch

        if not torch.cuda.is_available() or torch.version.hip:
            raise RuntimeError("The sm_100a kernels require an NVIDIA CUDA device")
        p = torch.cuda.get_device_properties(device)
        if p.major != 10:
            raise RuntimeError(
                f"Compute capability 10.x (B200, sm_100) required; device {device} is {p.major}.{p.minor}"
            )
        return cls(
            p.name,
            (p.major, p.minor),
            p.multi_processor_count,
            p.total_memory,
            getattr(p, "shared_memory_per_block_optin", p.shared_memory_per_block),
            getattr(p, "max_threads_per_block", 1024),
            getattr(p, "warp_size", 32),
            str(getattr(p, "uuid", "unknown")),
            device,
            nvlink_topology(device),
        )


def parse_topology(text):
    """Parse ``nvidia-smi topo -m`` output into {gpu_index: {peer_index: link}}.

    ``link`` is the matrix entry, e.g. ``NV18`` (18 NVLinks through NVSwitch),
    ``SYS``, ``PIX`` or ``X`` (self).  nvidia-smi underlines the header row with
    terminal escape sequences; they are removed before the columns are matched."""
    text = re.sub(r"\x1b\[[0-9;]*m", "", text)
    rows = [line.split() for line in text.splitlines() if line.strip()]
    if not rows:
        return {}
    header = [h for h in rows[0] if h.startswith("GPU")]
    topo = {}
    for row in rows[1:]:
        if not row or not row[0].startswith("GPU") or not row[0][3:].isdigit():
            continue
        gpu = int(row[0][3:])
        links = row[1 : 1 + len(header)]
        topo[gpu] = {int(h[3:]): link for h, link in zip(header, links) if h[3:].isdigit()}
    return topo


def nvlink_topology(device=0, runner=subprocess.run):
    """NVLink view of ``device``: peers, link label and NVLink count per peer.

    Uses ``nvidia-smi topo -m`` (read-only); falls back to an empty view when
    the tool is unavailable."""
    try:
        out = runner(["nvidia-smi", "topo", "-m"], capture_output=True, text=True, timeout=10).stdout
    except (OSError, subprocess.TimeoutExpired):
        return {}
    topo = parse_topology(out)
    mine = topo.get(device, {})
    peers = {}
    for peer, link in mine.items():
        if peer == device:
            continue
        count = int(link[2:]) if link.startswith("NV") and link[2:].isdigit() else 0
        peers[str(peer)] = {"link": link, "nvlinks": count}
    return {
        "gpus": len(topo),
        "peers": peers,
        "all_nvlink": bool(peers) and all(v["nvlinks"] > 0 for v in peers.values()),
    }


def gemm_shared_bytes(block_n, stages, experts=0):
    """Dynamic shared memory of the tcgen05 GEMM (csrc/gemm_tc.cuh gemm_tc_smem_bytes)."""
    a_bytes = GEMM_BM * GEMM_BK * 2
    b_bytes = block_n * GEMM_BK * 2
    total = 1024 + stages * (a_bytes + b_bytes) + EPILOGUE_BYTES + (2 * stages + 4) * 8 + 16
    if experts:
        total += (4 * experts + 4) * 4
    return total


def gemm_pair_shared_bytes(block_n, stages, experts=0):
    """Dynamic shared memory per CTA of the CTA-pair GEMM (csrc/gemm_tc2.cuh)."""
    return (1024 + stages * (GEMM_BM * GEMM_BK * 2 + (block_n // 2) * GEMM_BK * 2)
            + EPILOGUE_BYTES + (2 * stages + 4) * 8 + 16
            + ((4 * experts + 4) * 4 if experts else 0))


def rmsnorm_ring_bytes(columns, stages, elem_bytes=2):
    """Dynamic shared memory of the ring RMSNorm (csrc/rmsnorm.cuh rmsnorm_ring_smem_bytes)."""
    row = (columns * elem_bytes + 127) // 128 * 128
    return 128 + row * (stages + 1) + stages * 16 + 16


def resource_estimate(kernel, params, columns=0, experts=0):
    if kernel == "rmsnorm":
        threads = params["num_warps"] * 32
        rows = params["ROWS_PER_CTA"]
        per_row = max(threads // rows, 1)
        vectors = -(-(columns // 8) // per_row) if columns % 8 == 0 else 0
        stages = params.get("num_stages", 1)
        return {
            "threads_per_row": per_row,
            "vectors_per_thread": vectors,
            "single_pass_registers": vectors <= 16 and columns % 8 == 0,
            "shared_bytes_estimate": rmsnorm_ring_bytes(columns, stages) if stages >= 4 else 128,
        }
    return {
        "shared_bytes_estimate": gemm_shared_bytes(params["BLOCK_N"], params["num_stages"], experts),
        "accumulator_bytes": 4 * params["BLOCK_M"] * params["BLOCK_N"] * 2,
        "tmem_columns": 2 * params["BLOCK_N"],
    }


def prune_reason(hardware, kernel, params, columns=0, heuristic_smem=False):
    warps = params["num_warps"]
    if (
        warps not in (1, 2, 4, 8, 16, 32)
        and not (kernel != "rmsnorm" and warps == GEMM_WARPS)
    ) or warps * hardware.warp_size > hardware.max_threads_per_block:
        return "illegal_threads_per_block"
    if kernel == "rmsnorm":
        if params["ROWS_PER_CTA"] > warps * hardware.warp_size:
            return "rmsnorm_implementation_limit"
        stages = params.get("num_stages", 1)
        if stages >= 4 and columns % 8 == 0:
            # Ring kernel: each ring slot must always be consumed by the same warp.
            if stages % warps or (warps + 1) * hardware.warp_size > hardware.max_threads_per_block:
                return "rmsnorm_implementation_limit"
            if rmsnorm_ring_bytes(columns, stages) > hardware.shared_memory_per_block:
                return "shared_memory_exceeds_device_limit"
        return None
    if warps != GEMM_WARPS:
        return "illegal_threads_per_block"
    if params["BLOCK_M"] != GEMM_BM or params["BLOCK_K"] != GEMM_BK:
        return "illegal_tile_shape"
    if params["BLOCK_N"] not in (64, 128, 256) or 2 * params["BLOCK_N"] > TMEM_COLUMNS:
        return "illegal_tile_shape"
    pair = params.get("CTA_GROUP", 1) == 2
    if pair and params["BLOCK_N"] == 64:
        return "illegal_tile_shape"
    split = params.get("SPLIT_K", 1)
    if split < 1 or split > SPLIT_K_MAX or (split > 1 and pair and kernel == "moe_grouped_gemm"):
        return "illegal_split_k"
    experts = 64 if kernel == "moe_grouped_gemm" else 0
    smem = (gemm_pair_shared_bytes(params["BLOCK_N"], params["num_stages"], experts) if pair
            else gemm_shared_bytes(params["BLOCK_N"], params["num_stages"], experts))
    if smem > hardware.shared_memory_per_block:
        return "shared_memory_exceeds_device_limit"
    if heuristic_smem and smem > 0.85 * hardware.shared_memory_per_block:
        return "heuristic_shared_memory_estimate"
    return None

"""One categorical domain shared by Grid, Random and multivariate TPE, over CUDA launch parameters.

Same interface as the reference's ``bo_kernel_tuner/configs/search_spaces.py``
(``Workload`` :11-45, ``search_space`` :48-75, ``grid_size``/``grid_configs``
:78-83, ``validate_params`` :86-89).  The domains are redefined for the sm_100a
kernels:

* GEMM / MoE grouped GEMM: ``BLOCK_M`` is the tcgen05 MMA M (128 rows, one
  CTA); ``BLOCK_N`` the MMA N and TMEM accumulator width (x2 for double
  buffering); ``BLOCK_K`` one 128-byte swizzle row (64 elements);
  ``num_stages`` the depth of the TMA shared-memory ring; ``num_warps`` the
  warp-specialised CTA (TMA + MMA + 4 epilogue warps = 6); ``GROUP_M`` the
  grouped-M raster of the dense GEMM; ``CTA_MULTIPLIER`` the persistent grid
  of the grouped GEMM (``sm_count * CTA_MULTIPLIER``).
* ``CTA_GROUP`` 1 (one CTA per 128-row tile) or 2 (CTA pairs on two SMs,
  tcgen05 cta_group::2, 256-row tiles).  For the MoE grouped GEMM, 2 cuts each
  expert into 256-row pair tiles and a last block of at most 128 rows as a
  half-height pair tile (M = 128), so padding stays that of 128-row tiles.
* ``SPLIT_K`` 1 gives every tile one worker for its whole K loop (the
  reference's kernel, ``kernels/gemm.py:31-39``); S > 1 cuts each tile's K loop
  into S slices and deals the (tile, slice) units to the persistent CTAs in
  contiguous runs (split-K / stream-K).  With S < 4 (and in the grouped GEMM)
  the worker holding a tile's first slice adds the others' fp32 partials; a
  dense GEMM with S >= 4 stores every partial and sums them in a second,
  fully parallel kernel, so S up to 64 (tall-K shapes on all 148 SMs) stays
  cheap.  Single-CTA grouped tiles or dense tiles only (grouped CTA pairs are
  pruned).
* MoE grouped GEMM only: ``RASTER`` 1 walks the tiles expert by expert; 2 spreads
  the tiles of experts with at most two 128-row blocks (weights read once or
  twice: HBM-bound) evenly between the tiles of the others (tensor-bound).
* RMSNorm: ``ROWS_PER_CTA`` and ``num_warps`` as in the reference, plus
  ``num_stages``: 1 keeps the reference's one-row-slice-per-CTA shape; 2 (with
  ROWS_PER_CTA 1) a persistent CTA per resident slot that keeps its next row's
  loads in flight in a second register buffer; 4 or more the persistent kernel
  in which a producer warp streams rows into a ring of that many shared-memory
  row buffers (cp.async.bulk) and ``num_warps`` consumer warps normalise one
  row each.
"""

from dataclasses import asdict, dataclass
from itertools import product
from math import isfinite, prod

SPACE_VERSION = 4
KERNELS = ("gemm", "rmsnorm", "moe_grouped_gemm")


@dataclass(frozen=True)
class Workload:
    kernel: str = "gemm"
    m: int = 1024
    n: int = 1024
    k: int = 1024
    dtype: str = "fp16"
    expert_tokens: tuple[int, ...] = (64, 128, 256, 512)
    epsilon: float = 1e-6
    data_seed: int = 17

    def __post_init__(self):
        if self.kernel not in KERNELS or self.dtype not in ("fp16", "bf16"):
            raise ValueError("Unknown kernel or dtype")
        if min(self.m, self.n, self.k) <= 0 or not (isfinite(self.epsilon) and 0 < self.epsilon < 1):
            raise ValueError("Dimensions and epsilon must be positive; epsilon < 1")
        if not self.expert_tokens or min(self.expert_tokens) < 0 or sum(self.expert_tokens) <= 0:
            raise ValueError("Experts require nonnegative token counts and a positive total")
        if self.data_seed < 0:
            raise ValueError("data_seed must be nonnegative")

    def signature(self):
        """Only semantically relevant fields enter transfer compatibility."""
        d = asdict(self)
        if self.kernel == "rmsnorm":
            for key in ("k", "expert_tokens"):
                d.pop(key)
        else:
            d.pop("epsilon")
            if self.kernel == "gemm":
                d.pop("expert_tokens")
            else:
                d.pop("m")
                d["expert_tokens"] = list(self.expert_tokens)
        return d


def search_space(kernel: str, profile: str = "full") -> dict[str, list[int]]:
    if kernel not in KERNELS or profile not in ("full", "smoke"):
        raise ValueError("Unknown kernel or profile")
    if kernel == "rmsnorm":
        return {
            "ROWS_PER_CTA": [1, 2, 4, 8] if profile == "full" else [1, 2],
            "num_warps": [1, 2, 4, 8, 16] if profile == "full" else [4, 8],
            "num_stages": [1, 2, 4, 8, 16] if profile == "full" else [1, 2, 8],
        }
    space = {
        "BLOCK_M": [128],
        "BLOCK_N": [64, 128, 256],
        "BLOCK_K": [64],
        "num_warps": [6],
        "num_stages": [2, 3, 4, 5, 6],
    }
    if profile == "smoke":
        space = {
            "BLOCK_M": [128],
            "BLOCK_N": [64, 128],
            "BLOCK_K": [64],
            "num_warps": [6],
            "num_stages": [2],
        }
    if kernel == "gemm":
        space["GROUP_M"] = [1, 4, 8, 16] if profile == "full" else [1, 4]
        if profile == "full":
            space["CTA_GROUP"] = [1, 2]
    else:
        space["CTA_MULTIPLIER"] = [1, 2, 4] if profile == "full" else [1, 2]
        if profile == "full":
            space["RASTER"] = [1, 2]
            space["CTA_GROUP"] = [1, 2]
    if profile != "full":
        space["SPLIT_K"] = [1, 4]
    elif kernel == "gemm":
        space["SPLIT_K"] = [1, 2, 4, 8, 16, 32, 64]
    else:
        space["SPLIT_K"] = [1, 2, 4, 8, 16]
    return space


def default_params(kernel: str) -> dict[str, int]:
    """A good starting point on B200 (used by bench.py and as a tuning seed)."""
    if kernel == "rmsnorm":
        return {"ROWS_PER_CTA": 1, "num_warps": 4, "num_stages": 1}
    p = {"BLOCK_M": 128, "BLOCK_N": 256, "BLOCK_K": 64, "num_warps": 6, "num_stages": 4,
         "SPLIT_K": 1}
    if kernel == "gemm":
        p.update(GROUP_M=8, CTA_GROUP=2, num_stages=6)
    else:
        # CTA pairs (half-height tiles for short tails): 1,194 vs 975 TFLOP/s at 64 experts.
        p.update(CTA_MULTIPLIER=1, RASTER=1, CTA_GROUP=2, num_stages=6)
    return p


def grid_size(space):
    return prod(len(v) for v in space.values())


def grid_configs(space):
    return (dict(zip(space, values)) for values in product(*space.values()))


def validate_params(params, space):
    return set(params) == set(space) and all(
        type(params[k]) is int and params[k] in choices for k, choices in space.items()
    )

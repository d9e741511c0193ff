"""Seeded synthetic inputs for the benchmark configurations of the hot path.

Shapes and distributions of the five measured configurations:

* ``gemm_smoke``   C = A.B, 127 x 193 x 257 bf16, A, B ~ N(0, 1)
* ``rmsnorm``      x [4096, 4096] ~ N(0, 1), w [4096] ~ N(1, 0.1), bf16, eps 1e-6
* ``gemm``         square M = N = K (2048 or 8192), bf16/fp16, A, B ~ N(0, 1) * K^-0.5
* ``moe_small``    8 experts, W [8, 1024, 2048] ~ N(0, 0.02), token counts
                   [0, 16, 64, 256, 1024, 32, 8, 128], X [1528, 1024] ~ N(0, 1)
* ``moe_large``    64 experts, W [64, 4096, 14336] ~ N(0, 0.02), 16384 tokens
                   top-2 routed with Zipf(1.1) expert popularity, X [16384, 4096] ~ N(0, 1)

Every generator takes an explicit torch ``device`` and ``seed``; drawing on the
CPU gives the bit-identical inputs the CPU reference sees, drawing on the GPU
avoids a multi-GB host round trip for the large cases.  All data is synthetic:
the reference ships no dataset.
"""

import math

MOE_SMALL_COUNTS = (0, 16, 64, 256, 1024, 32, 8, 128)
MOE_SMALL = {"experts": 8, "k": 1024, "n": 2048}
MOE_LARGE = {"experts": 64, "k": 4096, "n": 14336, "tokens": 16384, "topk": 2, "zipf_s": 1.1}
RMSNORM = {"m": 4096, "n": 4096, "eps": 1e-6}
# RMSNorm of the 4096 x 4096 activations feeding a 4096 -> 14336 projection
# (the MoE expert shape): the fused norm-in-prologue GEMM.
RMSNORM_GEMM = {"m": 4096, "k": 4096, "n": 14336, "eps": 1e-6}


def _torch_dtype(dtype):
    import torch

    return {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]


def _gen(device, seed):
    import torch

    return torch.Generator(device=device).manual_seed(seed)


def gemm_inputs(m, n, k, dtype="bf16", seed=0, device="cpu", scaled=True):
    """A [m, k], B [k, n] ~ N(0, 1) (times k^-0.5 when ``scaled``)."""
    import torch

    g = _gen(device, seed)
    dt = _torch_dtype(dtype)
    a = torch.randn((m, k), generator=g, device=device, dtype=torch.float32)
    b = torch.randn((k, n), generator=g, device=device, dtype=torch.float32)
    if scaled:
        s = 1.0 / math.sqrt(k)
        a, b = a * s, b * s
    return a.to(dt), b.to(dt)


def rmsnorm_inputs(m=4096, n=4096, dtype="bf16", seed=0, device="cpu"):
    """x [m, n] ~ N(0, 1), w [n] ~ N(1, 0.1)."""
    import torch

    g = _gen(device, seed)
    dt = _torch_dtype(dtype)
    x = torch.randn((m, n), generator=g, device=device, dtype=torch.float32)
    w = 1.0 + 0.1 * torch.randn((n,), generator=g, device=device, dtype=torch.float32)
    return x.to(dt), w.to(dt)


def offsets_from_counts(counts):
    out = [0]
    for c in counts:
        out.append(out[-1] + int(c))
    return out


def moe_inputs(counts, k, n, dtype="bf16", seed=0, device="cpu", w_std=0.02):
    """X [sum(counts), k] ~ N(0, 1) packed in expert order, W [E, k, n] ~ N(0, w_std^2)."""
    import torch

    g = _gen(device, seed)
    dt = _torch_dtype(dtype)
    t = int(sum(counts))
    x = torch.randn((t, k), generator=g, device=device, dtype=torch.float32).to(dt)
    w = torch.empty((len(counts), k, n), device=device, dtype=dt)
    for e in range(len(counts)):  # per expert: bounds the fp32 temporary
        w[e] = (w_std * torch.randn((k, n), generator=g, device=device, dtype=torch.float32)).to(dt)
    return x, w


def zipf_probabilities(experts, s):
    """Expert popularity p_e proportional to (e + 1)^-s (expert 0 the hottest)."""
    import torch

    ranks = torch.arange(1, experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    return p / p.sum()


def zipf_routing(tokens, experts, topk=2, s=1.1, seed=0):
    """Top-k expert ids per token, drawn without replacement from Zipf(s)
    popularity with a seeded CPU generator; int32 [tokens, topk]."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    p = zipf_probabilities(experts, s).to(torch.float32)
    ids = torch.multinomial(p.expand(tokens, experts), topk, replacement=False, generator=g)
    return ids.to(torch.int32)


def moe_large_inputs(dtype="bf16", seed=0, device="cuda", tokens=None, experts=None, k=None,
                     n=None):
    """Token activations X [tokens, k], expert weights W [E, k, n] and the
    top-2 Zipf routing table (CPU-generated, so it is identical everywhere)."""
    import torch

    cfg = dict(MOE_LARGE)
    tokens = tokens or cfg["tokens"]
    experts = experts or cfg["experts"]
    k = k or cfg["k"]
    n = n or cfg["n"]
    ids = zipf_routing(tokens, experts, cfg["topk"], cfg["zipf_s"], seed)
    g = _gen(device, seed + 1)
    dt = _torch_dtype(dtype)
    x = torch.randn((tokens, k), generator=g, device=device, dtype=torch.float32).to(dt)
    w = torch.empty((experts, k, n), device=device, dtype=dt)
    for e in range(experts):
        w[e] = (0.02 * torch.randn((k, n), generator=g, device=device, dtype=torch.float32)).to(dt)
    return x, w, ids


def rmsnorm_gemm_inputs(m, k, n, dtype="bf16", seed=0, device="cpu"):
    """x [m, k] ~ N(0, 1), norm weight [k] ~ N(1, 0.1), B [k, n] ~ N(0, 1) * k^-0.5."""
    import torch

    x, w = rmsnorm_inputs(m, k, dtype, seed, device)
    g = _gen(device, seed + 1)
    b = torch.randn((k, n), generator=g, device=device, dtype=torch.float32) / math.sqrt(k)
    return x, w, b.to(_torch_dtype(dtype))

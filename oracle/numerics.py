"""FP32 references of the three kernels and the correctness gate, in numpy.

Test infrastructure only (see ``oracle/__init__.py``).  Inputs are float32
arrays holding the exact values of the fp16/bf16 operands; ``*_bits`` helpers
convert to and from the 16-bit storage formats.
"""

import numpy as np

TOLERANCES = {"fp16": (0.01, 0.02), "bf16": (0.02, 0.15)}  # reference worker.py:111
NORMWISE_LIMIT = 1e-2


# ----------------------------------------------------------------- 16-bit formats
def bf16_bits_to_f32(bits):
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    """Round-to-nearest-even float32 -> bfloat16 bits (NaN stays NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (u + (((u >> 16) & 1) + 0x7FFF)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def fp16_bits_to_f32(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_fp16_bits(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_f32(bits, dtype):
    return bf16_bits_to_f32(bits) if dtype == "bf16" else fp16_bits_to_f32(bits)


def from_f32(x, dtype):
    return f32_to_bf16_bits(x) if dtype == "bf16" else f32_to_fp16_bits(x)


def round_to(x, dtype):
    """Values of x after a cast to dtype (what a kernel's store produces)."""
    return to_f32(from_f32(x, dtype), dtype)


# ----------------------------------------------------------------- references
def gemm_fp32(a, b):
    """``a.float() @ b.float()`` (reference worker.py:64)."""
    return np.asarray(a, dtype=np.float32) @ np.asarray(b, dtype=np.float32)


def rmsnorm_fp32(x, weight, eps):
    """``x * rsqrt(mean(x^2, -1) + eps) * w`` in fp32 (reference worker.py:73-74)."""
    x = np.asarray(x, dtype=np.float32)
    mean_sq = np.mean(np.square(x), axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / np.sqrt(mean_sq + np.float32(eps))).astype(np.float32)
    return (x * inv) * np.asarray(weight, dtype=np.float32)


def rmsnorm_gemm_fp32(x, weight, b, eps):
    """The two-operator chain ``rmsnorm(x, w)`` (reference worker.py:73-74)
    followed by ``@ b`` (worker.py:64), in fp32 with no intermediate rounding:
    the answer the fused RMSNorm -> GEMM is gated against."""
    return gemm_fp32(rmsnorm_fp32(x, weight, eps), b)


def rmsnorm_row_scale_fp32(x, eps):
    """Per-row ``rsqrt(mean(x^2) + eps)`` in fp32: the factor rmsnorm_fp32
    multiplies each row by before the weight (reference worker.py:73-74)."""
    x = np.asarray(x, dtype=np.float32)
    mean_sq = np.mean(np.square(x), axis=-1, dtype=np.float32)
    return (np.float32(1.0) / np.sqrt(mean_sq + np.float32(eps))).astype(np.float32)


def grouped_gemm_fp32(x, weights, offsets):
    """Per-expert ``x[s_e:s_{e+1}] @ W[e]`` concatenated (reference worker.py:88-90).

    Rows outside [offsets[0], offsets[-1]) are returned as NaN: the operator
    does not write them."""
    x = np.asarray(x, dtype=np.float32)
    weights = np.asarray(weights, dtype=np.float32)
    out = np.full((x.shape[0], weights.shape[2]), np.nan, dtype=np.float32)
    for e in range(weights.shape[0]):
        s, t = int(offsets[e]), int(offsets[e + 1])
        if t > s:
            out[s:t] = x[s:t] @ weights[e]
    return out


# ----------------------------------------------------------------- gate
def check_output(out, reference, dtype):
    """The reference's gate (worker.py:108-116) plus the normwise relative error.

    Raises AssertionError like ``torch.testing.assert_close``."""
    rtol, atol = TOLERANCES[dtype]
    out = np.asarray(out, dtype=np.float32)
    reference = np.asarray(reference, dtype=np.float32)
    if out.shape != reference.shape:
        raise AssertionError(f"shape {out.shape} != {reference.shape}")
    if not np.isfinite(out).all() or not np.isfinite(reference).all():
        raise AssertionError("Nonfinite output or reference")
    delta = np.abs(out - reference)
    bad = delta > atol + rtol * np.abs(reference)
    if bad.any():
        idx = np.unravel_index(np.argmax(delta - (atol + rtol * np.abs(reference))), out.shape)
        raise AssertionError(
            f"{int(bad.sum())} / {out.size} elements outside rtol={rtol} atol={atol}; "
            f"worst at {idx}: out={out[idx]} ref={reference[idx]}"
        )
    rel = normwise_rel_error(out, reference)
    if rel > NORMWISE_LIMIT:
        raise AssertionError(f"normwise relative error {rel:.3e} > {NORMWISE_LIMIT}")
    return {
        "max_abs_error": float(delta.max()) if delta.size else 0.0,
        "normwise_rel_error": rel,
        "rtol": rtol,
        "atol": atol,
    }


def normwise_rel_error(out, reference):
    out = np.asarray(out, dtype=np.float64)
    reference = np.asarray(reference, dtype=np.float64)
    denom = np.linalg.norm(reference)
    return float(np.linalg.norm(out - reference) / denom) if denom > 0 else float(np.linalg.norm(out))

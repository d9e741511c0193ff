"""The reference's FP32 path as PyTorch expressions on CPU tensors — TEST INFRASTRUCTURE ONLY.

The timed CPU arm of ``bench.py`` (``cpu_baseline`` and ``--impl reference``)
runs these.  They are the reference worker's own FP32 formulas, written out
here because the reference package does not travel with this repository.
Each one consumes the 16-bit operands the way the reference does, converting
them with ``.float()`` inside the expression:

* GEMM: ``a.float() @ b.float()`` (``bo_kernel_tuner/tuner/worker.py:64``);
* RMSNorm: ``x.float() * rsqrt(mean(x.float()^2, -1) + eps)``, then ``* w.float()``
  (``worker.py:73-74``);
* MoE grouped GEMM: the concatenation over experts of
  ``x[s_e:s_{e+1}].float() @ W[e].float()`` (``worker.py:88-90``).

Intra-op threads come from ``configure``, i.e. ``torch.set_num_threads``.  FP32
matmul precision is set to "highest", as the reference's worker does
(``worker.py:171-174``).  ``configure`` also asks glibc to keep large freed
blocks in its heap: every call allocates fp32 temporaries of tens to hundreds
of MB, and by default each one is a fresh mapping that page-faults in, which
costs more than the arithmetic (4096 x 4096 RMSNorm: 0.9 GB/s with the default,
5.5-6 GB/s with reuse on 8 cores).  Correctness checks use the numpy
restatement in ``numerics``; this module only times the reference's own
formulation.
"""

import ctypes

import torch

_M_TRIM_THRESHOLD = -1
_M_MMAP_THRESHOLD = -3


def configure(threads):
    torch.set_num_threads(int(threads))
    torch.set_float32_matmul_precision("highest")
    try:
        libc = ctypes.CDLL("libc.so.6")
        libc.mallopt(_M_MMAP_THRESHOLD, ctypes.c_int(1 << 30))
        libc.mallopt(_M_TRIM_THRESHOLD, ctypes.c_int(2 ** 31 - 1))
    except OSError:  # not glibc: keep the allocator's defaults
        pass


def gemm(a, b):
    return a.float() @ b.float()


def rmsnorm(x, weight, eps):
    y = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + eps)
    return y * weight.float()


def grouped_gemm(x, weights, starts):
    return torch.cat([x[starts[e]:starts[e + 1]].float() @ weights[e].float()
                      for e in range(len(starts) - 1)])


def rmsnorm_gemm(x, weight, b, eps):
    """The two-call chain the fused kernel replaces, in the reference's formulas."""
    return gemm(rmsnorm(x, weight, eps), b)

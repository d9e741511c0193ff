"""CPU oracle for the bo-kernel-tuner hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the correctness reference or as the timed CPU reference.  The product path
(``flashattentionanycard_b200``) never imports it and has no CPU fallback.

Contents (numpy, fp32 arithmetic, restating the reference's FP32 path):

* ``numerics``: bf16/fp16 bit conversion, the FP32 references of the three
  kernels (reference ``bo_kernel_tuner/tuner/worker.py:64, 73-74, 88-90``) and
  the correctness gate (``worker.py:108-116``).
* ``reference_cpu``: the same FP32 formulas as PyTorch expressions on CPU
  tensors, as the reference's worker writes them; the timed CPU arm of
  ``bench.py`` runs these (never a checker).
* ``routing``: MoE expert histogram, offsets (``worker.py:83-86``), stable
  counting-sort permutation and inverse permutation (no reference counterpart;
  ``kernels/moe_grouped_gemm.py:3`` leaves routing outside the operator).

Pinning: ``tests/golden/`` holds vectors produced in the build container by
importing the reference itself — its FP32 formulas (``worker.prepare`` with the
``torch`` implementation on CPU) and its Triton kernels run under Triton's CPU
interpreter (fp16 GEMM / grouped GEMM, fp16 and bf16 RMSNorm; the interpreter's
bf16 ``tl.dot`` is unusable, so bf16 GEMM is pinned through the FP32 formula
only).  ``tests/test_oracle.py`` checks this oracle against every fixture.
Routing has no reference implementation: its parity is pinned to numpy's
stable argsort / bincount / cumsum, an independent formulation.
"""

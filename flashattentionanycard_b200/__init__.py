"""bo-kernel-tuner's hot path rebuilt for B200 (sm_100a).

``kernels/`` holds the drop-in ``launch`` functions of the reference's three
tuned kernels (GEMM, RMSNorm, MoE grouped GEMM) plus the device MoE routing
front end, all backed by the in-tree C-ABI library ``libbokt_sm100.so``;
``configs/`` and ``tuner/`` mirror the reference's search-space, hardware and
measurement-worker interfaces over the CUDA launch parameters; ``sharded``
partitions the paths that shard across GPUs.
"""

__version__ = "0.1.0"

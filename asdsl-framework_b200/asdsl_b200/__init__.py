"""asdsl_b200 -- B200-native (sm_100a) implementation of ASDSL's batch-1 W4A8
decode hot path: the preq / preq2 / Q4_128 / Q4_S256 / Q4_K GEMVs, the
UnifiedEngine decode step around them, and row-sharded projections over NCCL.

Submodules mirror the reference package layout for the path:
``asdsl_b200.kernels`` (asdsl.kernels), ``asdsl_b200.kernels._native_gemv``
(asdsl.kernels._native_gemv), ``asdsl_b200.kernels._native_unified``
(asdsl.kernels._native_unified), ``asdsl_b200.quantization`` (the offline
byte formats), ``asdsl_b200.sharding`` (multi-GPU row/K sharding).
"""

__version__ = "0.1.0"

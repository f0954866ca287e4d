"""fa_b200 -- B200 (sm_100a) flash-attention forward behind the platelett/fa
harness API.

Layout:
  csrc/      CUDA kernels (tcgen05 + TMA, warp-specialised) and the C ABI
  build.py   hash-keyed nvcc build of libb200fa.so
  lib.py     ctypes binding of the C ABI (include/b200fa.h)
  ops.py     torch-facing Operator (reference binding.py semantics)
  shard.py   multi-GPU partition of the (b, hq, q-block) unit grid
  core/      harness mirror: contract, registry, drivers, bench, runner,
             schedule, profiler (reference core/*)
  problem/   Case matrix and canonical inputs (reference problem/*)
  backends/  b200_fa_fp16, b200_fa_fp32 and the FP32 torch reference backend
"""

__all__ = ["ops", "lib", "build"]

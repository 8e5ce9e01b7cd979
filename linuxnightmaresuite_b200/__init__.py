"""B200-native mixture-of-experts layer forward.

A drop-in for the MoE FFN path of NightmareDesigns/Linuxnightmaresuite
(``moe_forward.py`` with GGUF Q4_0 / Q8_0 experts): router, dispatch, grouped
SwiGLU experts and combine run as hand-written sm_100a CUDA kernels in
``libmoe_b200.so``, called through a C ABI (include/moe_b200.h).

Modules:
  moe_forward  MoERouter / ExpertFFN / MoELayer / rms_norm (reference surface)
  kernels      torch-tensor wrappers of each C entry point
  ep           expert-parallel layer over NCCL all-to-all
  stacked      stacked decode step (MoE layers + shared expert + RMSNorm)
  synth        seeded synthetic workloads as raw GGUF block bytes
  build        nvcc build of the library
"""
__version__ = "1.0.0"

"""B200-native mixture-of-experts layer forward.

A drop-in for the MoE FFN path of NightmareDesigns/Linuxnightmaresuite
(``moe_forward.py`` and the streaming engines' MoE calls): router, dispatch,
grouped experts and combine run as hand-written sm_100a CUDA kernels in
``libmoe_b200.so``, called through a C ABI (include/moe_b200.h).

Modules:
  moe_forward  MoERouter / ExpertFFN / MoELayer / rms_norm (reference surface;
               GGUF block bytes or f32 matrices)
  kernels      torch-tensor wrappers of each C entry point
  gemma4       gemma4's MoE feed-forward block (GeGLU experts, fused gate_up,
               down scale, router input scale, sandwich norms)
  gguf         GGUF reader, expert-slice upload through pinned staging,
               whole-block loading
  engine       the reference engines' MoE calls served by the layer
  ep           expert parallelism over NVLink peer memory (IPC exchange
               windows, device-side send / serve / combine)
  stacked      stacked decode step (MoE layers + shared expert + RMSNorm)
  synth        seeded synthetic workloads as raw GGUF block bytes
  build        nvcc build of the library
"""
__version__ = "1.1.0"

"""fluidgpu_b200: B200-native (sm_100a) disaggregated decode step.

Host side in Python/PyTorch mirroring FluidGPU's runner / executor / comm /
KV-cache interfaces; compute in hand-written CUDA kernels behind the C ABI
of include/fgb200.h (libfgb200.so, built in-tree by fluidgpu_b200.build).
"""

__version__ = "0.1.0"

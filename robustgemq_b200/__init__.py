"""gemq-b200: B200-native (sm_100a) real-quant mixed-bit MoE expert path.

Drop-in for RobustGEMQ's quantized-MoE module API (``gemq.inference``) and its
kernel entry points (``gemq.triton_kernels``); every forward runs in the in-tree
``libgemq_b200.so`` (tcgen05 / TMA CUDA kernels behind a C ABI).
"""

__version__ = "0.1.0"

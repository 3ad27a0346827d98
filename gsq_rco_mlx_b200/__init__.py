"""B200-native (sm_100a) hot path of GSQ-RCO quantization.

Host code in Python keeps the module API of egesabanci/gsq-rco-mlx (gsq.gptq, gsq.lion,
gsq.staged, rco.manifold); every array computation runs in hand-written CUDA kernels of
libgsqrco_b200.so, called through its C ABI (include/gsq_rco_b200.h).
"""
__version__ = "0.1.0"

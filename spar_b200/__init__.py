"""spar_b200: B200-native (sm_100a) training backend for Spar's Transformer hot path.

The compute lives in libspar_b200.so (hand-written tcgen05/TMA GEMMs and fused bandwidth
kernels behind a C ABI, include/spar_b200.h and include/spar_cuda_kernels.h). This package only
binds it (ctypes) and provides host-side helpers; there is no CPU fallback.
"""
__version__ = "0.1.0"

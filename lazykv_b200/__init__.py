"""B200-native (sm_100a) implementation of LazyKV's tiered decode-attention hot path.

The modules mirror the reference's API for that path: `selection`, `quant`, `exact`, `tiered`,
`tiered_prefill`, `pinned`, `attention` and `cache`. Computation happens in hand-written CUDA
kernels in liblkv_sm100.so (C ABI in include/lkv.h), reached through `lazykv_b200._lib`.
"""

__version__ = "0.1.0"

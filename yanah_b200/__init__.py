"""B200 (sm_100a) sparse-MoE decode path for Yanah's moe_prefetch engine.

The CUDA kernels live in libyanah_b200.so (C ABI: include/yanah_b200.h);
this package holds the host side: record formats, synthetic workloads,
device weight holders, the resident stack decoder and the ModelBackend
implementation the reference orchestrator drives.
"""
__version__ = "0.1.0"

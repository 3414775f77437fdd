"""msplat (B200 build): the 2DGS training step on sm_100a behind a C ABI.

Mirrors the reference's Python surface (python/msplat/__init__.py):
TrainingConfig, TrainingStats, GaussianTrainer, sync, cleanup. The CUDA
library is libmsplat_b200.so (msplat-ios_b200/lib); nothing here falls back to
the CPU.
"""
__version__ = "0.1.0"

"""msplat (B200 build): the 2DGS training step on sm_100a behind a C ABI.

Mirrors the reference's Python surface (python/msplat/__init__.py):
TrainingConfig, TrainingStats, Dataset, GaussianTrainer, sync, cleanup and
load_dataset. The compute runs in libmsplat_b200.so (msplat-ios_b200/lib);
nothing here falls back to the CPU.
"""
from ._api import (Dataset, GaussianTrainer, TrainingConfig, TrainingStats, cleanup, load_dataset,  # noqa: F401
                   sync)

__all__ = ["TrainingConfig", "TrainingStats", "Dataset", "GaussianTrainer", "sync", "cleanup", "load_dataset"]

__version__ = "0.1.0"

"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (a B200 in this project) and exercise the
CUDA library through its C ABI; everything else runs on the CPU.
"""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "msplat-ios_b200", "python"), os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run with -m gpu)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")

"""Test configuration: the ``gpu`` marker and import paths.

Tests marked ``gpu`` need a B200 and the CUDA driver; everything else runs on
a CPU-only machine (lowering, NVRTC compilation to sm_100a, the oracle, the
host logic, the C-ABI exports).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")

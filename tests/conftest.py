"""Test configuration.

Markers:
  gpu -- needs a CUDA device (B200); deselect with -m "not gpu".
The repository root is put on sys.path so `cautreo_b200` (the product) and
`oracle` (the CPU checker) import from the working tree.
"""
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")

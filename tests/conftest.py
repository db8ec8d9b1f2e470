"""Shared pytest set-up: import paths and the ``gpu`` marker.

Tests marked ``gpu`` need a CUDA device and the built extension; everything
else runs on the CPU (``pytest -m "not gpu"``).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for path in (os.path.join(ROOT, "flash-spacetime_b200"), ROOT):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension"
    )

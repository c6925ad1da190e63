"""Shared pytest configuration.

Adds the package directory (``mlx-qsdpa_b200``) and the test oracle
(``oracle/``) to ``sys.path`` and registers the ``gpu`` and ``slow`` markers.
``-m "not gpu"`` runs everything that needs no CUDA device; ``-m gpu`` runs
the parity tests, which call the CUDA kernels through the C ABI.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("mlx-qsdpa_b200", "oracle", "tests"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libqsdpa.so")
    config.addinivalue_line("markers", "slow: long-running case")

"""Test configuration: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs the oracle, host-logic and C-ABI load tests (no GPU);
``-m gpu`` runs the parity tests proper on a CUDA device through the C ABI.
"""

import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "paged-attention-decode_b200"), os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200 / sm_100a)")

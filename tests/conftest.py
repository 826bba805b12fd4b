"""pytest configuration: markers and import paths.

``-m "not gpu"`` runs the CPU suite (oracle vs golden fixtures, oracle vs the
compiled reference, host-side planning logic, C-ABI exports, gloo multi-rank
tests).  ``-m gpu`` runs the parity tests of the CUDA path on a B200.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "ascend-spmm_b200"
for p in (ROOT, PKG, ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")

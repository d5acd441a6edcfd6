"""Shared pytest configuration.

Registers the ``gpu`` marker (tests that need a CUDA device) and puts the
repository root, the product package directory and tests/golden on
sys.path so tests import ``cuszp_wrapper_cpp``, ``oracle`` and ``cases``
the way users and the fixture script do.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "reducing-pcie-bottlenecks-for-llm-serving-with-cuszp-compressed-kv-cache-transfer_b200"
for p in (ROOT, PKG, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")

"""pytest configuration: the `gpu` marker and import paths.

Tests marked gpu need a B200 and the built libce_b200.so; everything else
runs on CPU (the oracle, host logic, gloo multi-process checks).
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libce_b200.so")

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


def pytest_sessionstart(session):
    """A fresh checkout has no libce_b200.so yet: compile it (nvcc for sm_100a,
    in-tree, as __graft_entry__.build does) before any test loads it.  An
    existing library is used as it is, so a test run never rebuilds what the
    build step made.  (The oracle builds itself on first use.)"""
    lib = ROOT / "cache_eviction_b200" / "_lib" / "libce_b200.so"
    if not lib.exists():
        from cache_eviction_b200 import build
        build.build(force=False)

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


GOLDEN = os.path.join(ROOT, "tests", "golden")


def reference_root():
    """The reference checkout, for the CPU tests that import its host code: QTTS_REFERENCE, or a
    directory named ``reference`` beside this repository; None when neither exists (the GPU box
    has no copy of it)."""
    from pathlib import Path
    cand = os.environ.get("QTTS_REFERENCE")
    paths = [Path(cand)] if cand else []
    paths.append(Path(ROOT).resolve().parent / "reference")
    for p in paths:
        if (p / "engine" / "backend" / "engine_loop.py").exists():
            return p
    return None

"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (the B200 parity tests); everything else
runs on CPU.  The product package lives in ``xllama-qwen35-xbox_b200/`` (a
directory name that is not a Python identifier), so its ``xq`` host package is
put on sys.path here; the oracle package sits at the repository root.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "xllama-qwen35-xbox_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 parity tests)")


def golden(name):
    import numpy as np
    return np.load(os.path.join(GOLDEN, name))

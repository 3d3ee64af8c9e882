"""Shared pytest setup: the ``gpu`` marker and import paths for the package and the oracle."""

from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "triton-attn_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built CUDA library")

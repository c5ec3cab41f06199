"""Shared pytest configuration.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``);
* puts the repository root (for ``oracle``) and the package root
  ``kv-cache-triton_b200`` (which holds the drop-in ``kernels`` / ``models`` /
  ``kvint4`` packages, laid out like the reference checkout) on ``sys.path``.
"""

from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kv-cache-triton_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")

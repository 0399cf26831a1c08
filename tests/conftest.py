"""Shared pytest configuration.

Markers: ``gpu`` tests need a B200 (run with ``-m gpu``); everything else runs on
the CPU. The oracle under ``oracle/`` is test infrastructure and is imported
here only as the checker.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()
# reference checkout (only this container's parity pins read it; GPU tests use the
# prebuilt oracle/_ref): $JADE_REFERENCE_ROOT, else "reference" beside this repository
REF_ROOT = os.environ.get("JADE_REFERENCE_ROOT") or os.path.join(os.path.dirname(ROOT), "reference")
HAS_REF = os.path.isdir(REF_ROOT)


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

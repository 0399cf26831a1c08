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
REF_ROOT = "/root/reference"
HAS_REF = os.path.isdir(REF_ROOT)


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

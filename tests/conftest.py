"""Shared pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 (sm_100) and the built library; everything
else runs on a CPU-only machine."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and libnf4b200.so")
    # tmp_path directories stay inside the checkout (git-ignored) unless the
    # caller chooses another place with --basetemp
    if config.option.basetemp is None:
        config.option.basetemp = str(ROOT / ".pytest_tmp")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

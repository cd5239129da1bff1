"""Test configuration: import paths and the `gpu` marker.

`-m "not gpu"` runs on any host: the oracle against the reference's golden vectors, host
logic, the C-ABI library's exports.  `-m gpu` is the parity suite on a B200: every call
goes through DecodeAttention -> libdory_decode.so (C ABI) -> the sm_100a kernel.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for sub in ("dory-vllm-experiments_b200", "oracle", "tests/golden", "tests", ""):
    path = str(ROOT / sub) if sub else str(ROOT)
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # GPU tests cannot run without a device; say so instead of failing on import.
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

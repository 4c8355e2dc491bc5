"""Shared test setup: import paths, the `gpu` marker, and the build step.

CPU tests (-m "not gpu") cover the oracle against known answers and golden
fixtures, the manager semantics on the bookkeeping backend, the C++ facade
and the exported C-ABI. GPU tests (-m gpu) are the parity tests proper: they
call libtllm_kv.so through its C-ABI and compare with the oracle.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tiny-llm_b200" / "python"))
sys.path.insert(0, str(ROOT / "tiny-llm_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_library():
    import build as tllm_build  # tiny-llm_b200/build.py
    import oracle as _oracle

    tllm_build.build_library()
    _oracle.build()
    yield


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False

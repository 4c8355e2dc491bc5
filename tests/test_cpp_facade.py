"""Runs the C++ facade test binary (reference KV tests ported to C++)."""
import subprocess

import pytest

import build as tllm_build
import conftest


def _run(*args):
    exe = tllm_build.build_cpp_tests()
    p = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    return p.stdout


def test_cpp_facade_bookkeeping():
    out = _run()
    assert "0 failed" in out


@pytest.mark.gpu
def test_cpp_facade_cuda():
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    out = _run("--gpu")
    assert "KVCacheAppendRetrieve" in out and "0 failed" in out

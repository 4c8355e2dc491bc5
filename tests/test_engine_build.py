"""The drop-in builds inside tiny-llm's own engine (CPU: compile and link only).

* Header swap alone: the reference's unpatched src/transformer.cpp and
  src/inference_engine.cpp compile with this repository's
  include/tiny_llm/kv_cache.h ahead of the engine's headers (the engine's
  types.h keeps its KVCacheConfig and result.h its Result<T>).
* The re-pointed engine: oracle/engine/drop_in.patch applies to the
  reference's sources, and the patched engine links against the C++ facade
  and libtllm_kv.so (oracle/Makefile.engine, which also builds the unpatched
  engine used as the baseline of tests/test_gpu_engine.py).
Skipped where the reference sources are not present (they are needed to
build, not to run).
"""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("TLLM_REFERENCE", "/root/reference"))


@pytest.fixture(autouse=True)
def _need_reference():
    if not (REF / "src" / "transformer.cpp").exists():
        pytest.skip("reference sources not present")


def _make(*targets):
    p = subprocess.run(["make", "-s", "-j8", "-C", str(ROOT / "oracle"), "-f", "Makefile.engine",
                        f"REF={REF}", *targets], capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stdout[-4000:] + p.stderr[-4000:]


def test_engine_sources_compile_against_the_drop_in_header():
    _make("syntax")


def test_patched_engine_links_against_the_paged_cache():
    _make("all")
    for exe in ("engine_ref", "engine_dropin"):
        assert (ROOT / "oracle" / "_ref" / "engine" / exe).exists()
    nm = subprocess.run(["nm", "-C", "--undefined-only", str(ROOT / "oracle" / "_ref" / "engine" / "engine_dropin")],
                        capture_output=True, text=True).stdout
    # the engine calls the C-ABI; the reference's own KVCacheManager is not in it
    assert "tl_decode_attention" in nm and "tl_prefill_attention" in nm
    defined = subprocess.run(["nm", "-C", "--defined-only", str(ROOT / "oracle" / "_ref" / "engine" / "engine_dropin")],
                             capture_output=True, text=True).stdout
    assert "tiny_llm::KVCacheManager::decodeAttention" in defined
    assert "tiny_llm::TransformerLayer::forwardBatch" in defined

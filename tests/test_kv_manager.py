"""KV cache manager semantics through the C-ABI, on the bookkeeping backend.

Each test ports one behaviour of the reference's tests/test_kv_cache.cpp
(line numbers in the docstrings) or covers a paged-pool behaviour that the
block allocator adds (growth, free-list reuse, block exhaustion, rollback).
The bookkeeping backend keeps the pool in host memory and refuses every call
that would launch a kernel, so these run without a GPU.
"""
import re
from pathlib import Path

import pytest

import tiny_llm_b200 as T

BK = T.TL_BACKEND_HOST_BOOKKEEPING
ROOT = Path(__file__).resolve().parents[1]


def make(num_layers=2, num_heads=4, head_dim=64, max_seq_len=128, max_batch_size=4, **kw):
    return T.KVCache(num_layers=num_layers, num_kv_heads=num_heads, head_dim=head_dim,
                     max_seq_len=max_seq_len, max_batch_size=max_batch_size, backend=BK, **kw)


def test_library_exports_every_declared_symbol():
    lib = T.load()
    declared = set()
    for h in (ROOT / "include").glob("*.h"):
        declared |= set(re.findall(r"\b(tl_[a-z0-9_]+)\s*\(", h.read_text()))
    assert declared, "no declarations found"
    assert declared == set(T.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.tl_version()


def test_initialization_allocates_memory():  # test_kv_cache.cpp:43-51
    c = make()
    assert c.total_memory() > 0
    assert c.used_memory() == 0
    assert c.active_sequence_count() == 0


def test_allocate_returns_valid_id():  # :53-65
    c = make()
    sid = c.allocate_sequence(64)
    assert sid >= 0 and c.has_sequence(sid) and c.get_seq_len(sid) == 0


def test_allocate_multiple_unique_ids():  # :67-85
    c = make(max_batch_size=4)
    ids = [c.allocate_sequence(64) for _ in range(4)]
    assert c.active_sequence_count() == 4 and len(set(ids)) == 4


def test_exhaustion_returns_error():  # :87-100
    c = make(max_batch_size=2)
    c.allocate_sequence(64)
    c.allocate_sequence(64)
    with pytest.raises(T.Exhausted) as e:
        c.allocate_sequence(64)
    assert "exhausted" in str(e.value)


def test_release_frees_slot():  # :102-122
    c = make(max_batch_size=2)
    s1 = c.allocate_sequence(64)
    c.allocate_sequence(64)
    c.release_sequence(s1)
    assert not c.has_sequence(s1) and c.active_sequence_count() == 1
    s3 = c.allocate_sequence(64)
    assert s3 not in (s1,)  # ids are never reused (kv_cache.cpp:110)


def test_release_unknown_is_not_found():
    c = make()
    with pytest.raises(T.NotFound) as e:
        c.release_sequence(12345)
    assert "not found" in str(e.value)


def test_get_cache_valid_pointers():  # :124-139
    c = make()
    sid = c.allocate_sequence(64)
    for layer in range(2):
        k, v = c.get_cache(sid, layer)
        assert k and v and k != v


def test_get_cache_invalid_sequence_is_null():  # :141-149
    c = make()
    assert c.get_cache(999, 0) == (None, None)


def test_invalid_max_len():  # :151-167
    c = make(max_seq_len=128)
    for bad in (0, -1, 256):
        with pytest.raises(T.InvalidArgument) as e:
            c.allocate_sequence(bad)
        assert "Invalid max_len" in str(e.value)


def test_memory_accounting():  # :169-194
    c = make()
    total = c.total_memory()
    assert c.free_memory() == total and c.used_memory() == 0
    c.allocate_sequence(64)
    one = c.used_memory()
    assert one > 0 and c.free_memory() == total - one
    c.allocate_sequence(64)
    assert c.used_memory() == 2 * one


def test_invalid_layer_is_null():  # :227-243
    c = make(2, 4, 8, 32, 2)
    sid = c.allocate_sequence(16)
    assert c.get_cache(sid, -1) == (None, None)
    assert c.get_cache(sid, 2) == (None, None)
    with pytest.raises(T.InvalidArgument) as e:
        c.get_cache_checked(sid, 2)
    assert "Invalid layer_idx" in str(e.value)


def test_invalid_appends_do_not_advance():  # :245-260
    c = make(2, 4, 8, 32, 2)
    sid = c.allocate_sequence(16)
    with pytest.raises(T.InvalidArgument):
        c.append_kv(sid, -1, None, None, 0)
    with pytest.raises(T.InvalidArgument) as e:
        c.append_kv(sid, 2, None, None, 1)
    assert "is null" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        c.append_kv(sid, 0, 16, 16, 0)
    assert "must be positive" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        c.append_kv(sid, 5, 16, 16, 1)
    assert "Invalid layer_idx" in str(e.value)
    with pytest.raises(T.NotFound):
        c.append_kv(777, 0, 16, 16, 1)
    with pytest.raises(T.Overflow) as e:
        c.append_kv(sid, 0, 16, 16, 17)
    assert "overflow" in str(e.value)
    assert c.get_seq_len(sid) == 0


def test_append_on_bookkeeping_backend_refuses_compute():
    c = make(2, 4, 64, 32, 2)
    sid = c.allocate_sequence(16)
    with pytest.raises(T.NoDevice):
        c.append_kv(sid, 0, 16, 16, 1)
    with pytest.raises(T.NoDevice):
        c.decode_attention(0, 16, 16, [sid])
    assert c.get_seq_len(sid) == 0


def test_attention_step_validates_then_refuses_compute():
    """tl_attention_step: argument errors as appendKV / decodeAttention report
    them; on the bookkeeping backend it refuses before touching any state."""
    c = make(2, 4, 64, 32, 2)
    sid = c.allocate_sequence(16)
    with pytest.raises(T.InvalidArgument) as e:
        c.attention_step(2, 16, 16, 16, 16, [sid])
    assert "Invalid layer_idx" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        c.attention_step(0, None, 16, 16, 16, [sid])
    assert "query is null" in str(e.value)
    with pytest.raises(T.NotFound):
        c.attention_step(0, 16, 16, 16, 16, [sid + 99])
    with pytest.raises(T.InvalidArgument) as e:
        c.attention_step(0, 16, 16, 16, 16, [sid, sid])
    assert "duplicate" in str(e.value)
    with pytest.raises(T.NoDevice):
        c.attention_step(0, 16, 16, 16, 16, [sid])
    assert c.get_seq_len(sid) == 0
    assert c.pool_stats().used_blocks == 1  # the block taken at allocation, nothing grown


def test_prefill_attention_validates_arguments():
    """tl_prefill_attention: bad layer, null pointers, unknown or duplicate
    sequences, and query counts outside [1, written tokens] are refused."""
    c = make(2, 4, 64, 32, 2)
    sid = c.allocate_sequence(16)
    with pytest.raises(T.InvalidArgument) as e:
        c.prefill_attention(5, 16, 16, [sid], [1])
    assert "Invalid layer_idx" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        c.prefill_attention(0, None, 16, [sid], [1])
    assert "query is null" in str(e.value)
    with pytest.raises(T.NotFound):
        c.prefill_attention(0, 16, 16, [sid + 5], [1])
    with pytest.raises(T.InvalidArgument) as e:
        c.prefill_attention(0, 16, 16, [sid, sid], [1, 1])
    assert "duplicate" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:  # nothing written yet
        c.prefill_attention(0, 16, 16, [sid], [1])
    assert "num_tokens must be in" in str(e.value)
    with pytest.raises(T.InvalidArgument):
        c.prefill_attention(0, 16, 16, [sid], [1, 2])


def test_project_qkv_append_validates_arguments():
    """tl_project_qkv_append: bad layer, null pointers, shapes outside the
    kernel's (hidden not a multiple of 128, group sizes other than
    16/32/64/128), misalignment, unknown/duplicate sequences and a full
    sequence are refused before any device work; the bookkeeping backend
    then reports that it has no device."""
    c = make(2, 4, 64, 32, 2)
    sid = c.allocate_sequence(2)
    ok = dict(x=16, hidden=256, wq=16, sq=16, wk=16, sk=16, wv=16, sv=16, group=32, sids=[sid], q=16)

    def call(layer=0, **kw):
        a = dict(ok, **kw)
        c.project_qkv_append(layer, a["x"], a["hidden"], a["wq"], a["sq"], a["wk"], a["sk"], a["wv"], a["sv"],
                             a["group"], a["sids"], a["q"])

    with pytest.raises(T.InvalidArgument) as e:
        call(layer=2)
    assert "Invalid layer_idx" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        call(x=None)
    assert "input is null" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        call(q=None)
    assert "q output is null" in str(e.value)
    with pytest.raises(T.InvalidArgument):
        call(wk=None)
    with pytest.raises(T.InvalidArgument):
        call(hidden=0)
    with pytest.raises(T.Unsupported):
        call(hidden=200)
    with pytest.raises(T.Unsupported):
        call(group=8)
    with pytest.raises(T.InvalidArgument) as e:
        call(sq=18)
    assert "aligned" in str(e.value)
    with pytest.raises(T.NotFound):
        call(sids=[sid + 7])
    with pytest.raises(T.InvalidArgument) as e:
        call(sids=[sid, sid])
    assert "duplicate" in str(e.value)
    with pytest.raises(T.NoDevice):
        call()
    c.advance_seq_len(sid, 2)
    with pytest.raises(T.Overflow) as e:
        call()
    assert "overflow" in str(e.value)
    call(sids=[])  # nothing to do


def test_project_qkv_append_packed_validates_arguments():
    """tl_project_qkv_append_packed runs the same checks (under its own
    name) before any device work, and tl_qkv_pack_weight refuses null,
    misaligned and overlapping buffers and widths outside multiples of 128
    before it looks for a device."""
    c = make(2, 4, 64, 32, 2)
    sid = c.allocate_sequence(2)

    def call(layer=0, x=16, hidden=256, group=32, sids=(sid,)):
        c.project_qkv_append_packed(layer, x, hidden, 16, 16, 16, 16, 16, 16, group, list(sids), 16)

    with pytest.raises(T.InvalidArgument) as e:
        call(layer=5)
    assert "projectQKVAppendPacked" in str(e.value)
    with pytest.raises(T.InvalidArgument):
        call(x=None)
    with pytest.raises(T.Unsupported):
        call(hidden=200)
    with pytest.raises(T.NotFound):
        call(sids=(sid + 3,))
    with pytest.raises(T.NoDevice):
        call()
    call(sids=())

    with pytest.raises(T.InvalidArgument) as e:
        T.pack_qkv_weight(None, 256, 128, 1 << 20)
    assert "null" in str(e.value)
    with pytest.raises(T.Unsupported):
        T.pack_qkv_weight(1 << 20, 200, 128, 1 << 24)
    with pytest.raises(T.Unsupported):
        T.pack_qkv_weight(1 << 20, 256, 96, 1 << 24)
    with pytest.raises(T.InvalidArgument) as e:
        T.pack_qkv_weight((1 << 20) + 4, 256, 128, 1 << 24)
    assert "aligned" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        T.pack_qkv_weight(1 << 20, 256, 128, (1 << 20) + 256 * 64)
    assert "overlap" in str(e.value)


def test_advance_clamps_to_capacity():  # :262-273
    c = make(2, 4, 8, 32, 2)
    sid = c.allocate_sequence(5)
    c.advance_seq_len(sid, 100)
    assert c.get_seq_len(sid) == 5


def test_advance_ignores_non_positive():  # :275-287
    c = make(2, 4, 8, 32, 2)
    sid = c.allocate_sequence(5)
    for n in (0, -3):
        with pytest.raises(T.InvalidArgument):
            c.advance_seq_len(sid, n)
    assert c.get_seq_len(sid) == 0


def test_multiple_sequences_independent():  # test_integration.cu:173-205
    c = make(2, 4, 16, 32, 4)
    ids = [c.allocate_sequence(16) for _ in range(3)]
    assert len(set(ids)) == 3
    for s in ids:
        c.release_sequence(s)
    assert c.active_sequence_count() == 0 and c.used_memory() == 0


# ---- paged-pool behaviour ---------------------------------------------------

def test_blocks_grow_with_length_and_return_on_release():
    c = make(2, 2, 64, 100, 4, block_size=16)
    sid = c.allocate_sequence(100)
    assert len(c.block_table(sid)) == 1
    c.advance_seq_len(sid, 33)
    assert len(c.block_table(sid)) == 3  # ceil(33/16)
    c.reserve(sid, 80)
    assert len(c.block_table(sid)) == 5
    st = c.pool_stats()
    assert st.used_blocks == 5 and st.high_water == 5
    c.release_sequence(sid)
    st = c.pool_stats()
    assert st.used_blocks == 0 and st.free_blocks == st.num_blocks


def test_free_list_reuse_is_lifo():
    c = make(1, 1, 64, 64, 4)
    a = c.allocate_sequence(64)
    b = c.allocate_sequence(64)
    ba = c.block_table(a)
    c.release_sequence(a)
    d = c.allocate_sequence(64)
    assert c.block_table(d) == ba  # the block just released is reused first
    assert c.block_table(b) != ba


def test_block_exhaustion_rolls_back():
    c = make(1, 1, 64, 64, 4, num_blocks=5)  # 5 blocks of 16 tokens
    a = c.allocate_sequence(64)
    c.reserve(a, 64)  # 4 blocks
    b = c.allocate_sequence(64)  # the 5th
    used = c.pool_stats().used_blocks
    with pytest.raises(T.Exhausted) as e:
        c.reserve(b, 40)  # needs 3, only 0 free
    assert "exhausted" in str(e.value)
    assert c.pool_stats().used_blocks == used
    assert len(c.block_table(b)) == 1
    with pytest.raises(T.Exhausted):
        c.allocate_sequence(10)  # a slot is free but no block is
    assert c.active_sequence_count() == 2


def test_reserve_beyond_max_len_is_overflow():
    c = make(1, 1, 64, 64, 2)
    s = c.allocate_sequence(20)
    with pytest.raises(T.Overflow):
        c.reserve(s, 21)


def test_permuted_free_list_is_a_permutation():
    c = make(1, 1, 64, 64, 8, num_blocks=32)
    c.permute_free_blocks(1234)
    got = []
    ids = [c.allocate_sequence(64) for _ in range(8)]
    for s in ids:
        c.reserve(s, 64)
        got += c.block_table(s)
    assert sorted(got) == list(range(32)) and got != list(range(32))


def test_invalid_configs_rejected():
    for kw in (dict(num_layers=0), dict(num_heads=0), dict(head_dim=0), dict(max_seq_len=0),
               dict(max_batch_size=0)):
        with pytest.raises(T.InvalidArgument) as e:
            make(**kw)
        assert "invalid configuration" in str(e.value)
    with pytest.raises(T.InvalidArgument):
        make(block_size=24)
    with pytest.raises(T.InvalidArgument):
        make(num_heads=4, num_q_heads=6)


def test_size_overflow_detected():
    with pytest.raises(T.Overflow) as e:
        make(num_layers=1 << 20, num_heads=1 << 12, head_dim=1 << 12, max_seq_len=1 << 20,
             max_batch_size=1 << 10)
    assert "overflow" in str(e.value)


def test_injected_allocation_failure_is_reported_and_clean():
    T.inject_alloc_failure(1)
    try:
        with pytest.raises(T.CudaError) as e:
            make()
        assert "injected" in str(e.value)
    finally:
        T.inject_alloc_failure(0)
    c = make()  # next create works
    assert c.total_memory() > 0


def test_cuda_backend_without_device_fails_loudly():
    import conftest
    if conftest.cuda_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(T.NoDevice) as e:
        T.KVCache(num_layers=1, num_kv_heads=1, head_dim=64, max_seq_len=16)
    assert "no CUDA device" in str(e.value)


def test_rope_table_matches_oracle_bitwise():
    import numpy as np
    import oracle as O
    c1, s1 = T.rope_table(257, 128, 10000.0)
    c2, s2 = O.rope_table(257, 128, 10000.0)
    assert np.array_equal(c1.view(np.uint32), c2.view(np.uint32))
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32))

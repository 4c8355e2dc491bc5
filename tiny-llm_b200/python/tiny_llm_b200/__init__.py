"""ctypes binding of libtllm_kv.so (include/tllm_kv.h).

Mirrors the reference's KVCacheManager interface (AICL-Lab/tiny-llm
include/tiny_llm/kv_cache.h:24-111) in Python for the tests and the bench:
the same operations, argument meaning and error behaviour, with C-ABI status
codes raised as TLError subclasses whose messages carry the reference's
error texts. Device buffers are passed as integer addresses (for example
torch.Tensor.data_ptr()); streams as integer handles (cuda_stream).

There is no CPU fallback: if the shared library is missing, load() raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG_ROOT = Path(__file__).resolve().parents[2]  # tiny-llm_b200/
LIB_PATH = _PKG_ROOT / "lib" / "libtllm_kv.so"

TL_OK = 0
TL_ERR_INVALID_ARG = -1
TL_ERR_NOT_FOUND = -2
TL_ERR_EXHAUSTED = -3
TL_ERR_OVERFLOW = -4
TL_ERR_CUDA = -5
TL_ERR_NO_DEVICE = -6
TL_ERR_UNSUPPORTED = -7
TL_ERR_DEVICE_FAULT = -8

TL_BACKEND_CUDA = 0
TL_BACKEND_HOST_BOOKKEEPING = 1
TL_LAYOUT_TOKEN_MAJOR = 0
TL_LAYOUT_HEAD_MAJOR = 1

# Every symbol include/tllm_kv.h declares (checked by the CPU tests).
EXPORTED_SYMBOLS = [
    "tl_config_init", "tl_create", "tl_destroy", "tl_last_error", "tl_status_name",
    "tl_allocate_sequence", "tl_release_sequence", "tl_reserve", "tl_get_cache",
    "tl_append_kv", "tl_append_kv_all_layers", "tl_advance_seq_len", "tl_get_seq_len",
    "tl_has_sequence", "tl_used_memory", "tl_total_memory", "tl_free_memory",
    "tl_active_sequence_count", "tl_get_config", "tl_get_block_table", "tl_get_pool_stats",
    "tl_get_pool", "tl_decode_attention", "tl_sync_check", "tl_rope_table",
    "tl_permute_free_blocks", "tl_debug_inject_alloc_failure", "tl_version",
    "tl_decode_attention_static", "tl_peer_init", "tl_peer_connect", "tl_peer_buffer",
    "tl_decode_attention_peer", "tl_attention_step", "tl_prefill_attention",
    "tl_project_qkv_append", "tl_sample_tokens", "tl_set_peer_wait_limit", "tl_debug_peer_attach",
    "tl_qkv_pack_weight", "tl_project_qkv_append_packed",
]


class TLError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class InvalidArgument(TLError): pass
class NotFound(TLError): pass
class Exhausted(TLError): pass
class Overflow(TLError): pass
class CudaError(TLError): pass
class NoDevice(TLError): pass
class Unsupported(TLError): pass
class DeviceFault(TLError): pass


_ERRORS = {
    TL_ERR_INVALID_ARG: InvalidArgument, TL_ERR_NOT_FOUND: NotFound,
    TL_ERR_EXHAUSTED: Exhausted, TL_ERR_OVERFLOW: Overflow, TL_ERR_CUDA: CudaError,
    TL_ERR_NO_DEVICE: NoDevice, TL_ERR_UNSUPPORTED: Unsupported,
    TL_ERR_DEVICE_FAULT: DeviceFault,
}


class Config(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int), ("num_kv_heads", C.c_int), ("head_dim", C.c_int),
        ("max_seq_len", C.c_int), ("max_batch_size", C.c_int), ("block_size", C.c_int),
        ("num_blocks", C.c_longlong), ("num_q_heads", C.c_int), ("rope_theta", C.c_float),
        ("rope_on_append", C.c_int), ("layout", C.c_int), ("backend", C.c_int),
        ("device", C.c_int),
    ]


class PagedView(C.Structure):
    """tl_paged_view: a caller-owned pool for tl_decode_attention_static."""
    _fields_ = [
        ("pool", C.c_void_p), ("block_tables", C.c_void_p), ("error_word", C.c_void_p),
        ("num_blocks", C.c_longlong), ("num_layers", C.c_int), ("num_kv_heads", C.c_int),
        ("num_q_heads", C.c_int), ("head_dim", C.c_int), ("block_size", C.c_int),
        ("layout", C.c_int), ("bt_stride", C.c_int), ("num_rows", C.c_int),
    ]


class PoolStats(C.Structure):
    _fields_ = [
        ("num_blocks", C.c_longlong), ("used_blocks", C.c_longlong),
        ("free_blocks", C.c_longlong), ("high_water", C.c_longlong),
        ("block_bytes", C.c_longlong), ("active_sequences", C.c_int),
        ("max_blocks_per_seq", C.c_int), ("kernel_launches", C.c_longlong),
    ]


_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Loads libtllm_kv.so (building is __graft_entry__.build()'s job)."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(
            f"{p} is missing: build it with `python __graft_entry__.py build` "
            "(there is no CPU fallback for this library)")
    lib = C.CDLL(str(p))
    vp, i, f, ll, sz = C.c_void_p, C.c_int, C.c_float, C.c_longlong, C.c_size_t
    ip = C.POINTER(C.c_int)
    sigs = {
        "tl_config_init": (None, [C.POINTER(Config)]),
        "tl_create": (i, [C.POINTER(Config), C.POINTER(vp)]),
        "tl_destroy": (None, [vp]),
        "tl_last_error": (C.c_char_p, [vp]),
        "tl_status_name": (C.c_char_p, [i]),
        "tl_allocate_sequence": (i, [vp, i, ip]),
        "tl_release_sequence": (i, [vp, i]),
        "tl_reserve": (i, [vp, i, i]),
        "tl_get_cache": (i, [vp, i, i, C.POINTER(vp), C.POINTER(vp)]),
        "tl_append_kv": (i, [vp, i, i, vp, vp, i, vp]),
        "tl_append_kv_all_layers": (i, [vp, ip, i, vp, vp, vp]),
        "tl_advance_seq_len": (i, [vp, i, i]),
        "tl_get_seq_len": (i, [vp, i]),
        "tl_has_sequence": (i, [vp, i]),
        "tl_used_memory": (sz, [vp]),
        "tl_total_memory": (sz, [vp]),
        "tl_free_memory": (sz, [vp]),
        "tl_active_sequence_count": (i, [vp]),
        "tl_get_config": (i, [vp, C.POINTER(Config)]),
        "tl_get_block_table": (i, [vp, i, ip, i, ip]),
        "tl_get_pool_stats": (i, [vp, C.POINTER(PoolStats)]),
        "tl_get_pool": (i, [vp, C.POINTER(vp), C.POINTER(sz)]),
        "tl_decode_attention": (i, [vp, i, vp, vp, ip, i, f, vp]),
        "tl_attention_step": (i, [vp, i, vp, vp, vp, vp, ip, i, f, vp]),
        "tl_prefill_attention": (i, [vp, i, vp, vp, ip, ip, i, f, vp]),
        "tl_project_qkv_append": (i, [vp, i, vp, i, vp, vp, vp, vp, vp, vp, i, ip, i, vp, vp]),
        "tl_project_qkv_append_packed": (i, [vp, i, vp, i, vp, vp, vp, vp, vp, vp, i, ip, i, vp, vp]),
        "tl_qkv_pack_weight": (i, [vp, i, i, vp, vp]),
        "tl_sample_tokens": (i, [vp, ll, i, i, i, f, i, f, C.c_ulonglong, C.c_ulonglong, vp, vp]),
        "tl_sync_check": (i, [vp, vp]),
        "tl_rope_table": (None, [C.POINTER(C.c_float), C.POINTER(C.c_float), i, i, f]),
        "tl_permute_free_blocks": (i, [vp, C.c_ulonglong]),
        "tl_debug_inject_alloc_failure": (i, [i]),
        "tl_version": (C.c_char_p, []),
        "tl_decode_attention_static": (i, [C.POINTER(PagedView), i, vp, vp, ip, ip, i, f, vp,
                                           C.c_char_p, i]),
        "tl_peer_init": (i, [vp, i, i, sz, vp]),
        "tl_peer_connect": (i, [vp, vp]),
        "tl_peer_buffer": (i, [vp, C.POINTER(vp), C.POINTER(sz)]),
        "tl_decode_attention_peer": (i, [vp, i, vp, ip, i, f, sz, C.c_uint, vp]),
        "tl_set_peer_wait_limit": (i, [vp, C.c_double]),
        "tl_debug_peer_attach": (i, [vp, i, vp]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _ids(seq_ids):
    arr = (C.c_int * len(seq_ids))(*[int(s) for s in seq_ids])
    return arr


class KVCache:
    """The paged KV cache handle (KVCacheManager equivalent)."""

    def __init__(self, num_layers=32, num_kv_heads=32, head_dim=128, max_seq_len=2048,
                 max_batch_size=1, block_size=16, num_blocks=0, num_q_heads=0,
                 rope_theta=10000.0, rope_on_append=False, layout=TL_LAYOUT_TOKEN_MAJOR,
                 backend=TL_BACKEND_CUDA, device=-1):
        self._lib = load()
        cfg = Config()
        self._lib.tl_config_init(C.byref(cfg))
        cfg.num_layers, cfg.num_kv_heads, cfg.head_dim = num_layers, num_kv_heads, head_dim
        cfg.max_seq_len, cfg.max_batch_size = max_seq_len, max_batch_size
        cfg.block_size, cfg.num_blocks, cfg.num_q_heads = block_size, num_blocks, num_q_heads
        cfg.rope_theta, cfg.rope_on_append = rope_theta, int(bool(rope_on_append))
        cfg.layout, cfg.backend, cfg.device = layout, backend, device
        h = C.c_void_p()
        st = self._lib.tl_create(C.byref(cfg), C.byref(h))
        if st != TL_OK:
            msg = self._lib.tl_last_error(None).decode()
            raise _ERRORS.get(st, TLError)(st, msg)
        self._h = h
        got = Config()
        self._lib.tl_get_config(self._h, C.byref(got))
        self.config = got

    # -- lifecycle ---------------------------------------------------------
    def close(self):
        if getattr(self, "_h", None):
            self._lib.tl_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, st):
        if st != TL_OK:
            msg = self._lib.tl_last_error(self._h).decode()
            raise _ERRORS.get(st, TLError)(st, msg)

    # -- reference API -----------------------------------------------------
    def allocate_sequence(self, max_len: int) -> int:
        sid = C.c_int(-1)
        self._check(self._lib.tl_allocate_sequence(self._h, int(max_len), C.byref(sid)))
        return sid.value

    def release_sequence(self, seq_id: int) -> None:
        self._check(self._lib.tl_release_sequence(self._h, int(seq_id)))

    def reserve(self, seq_id: int, new_len: int) -> None:
        self._check(self._lib.tl_reserve(self._h, int(seq_id), int(new_len)))

    def get_cache(self, seq_id: int, layer: int):
        """getCache: (k_ptr, v_ptr), (None, None) on error like the reference."""
        k, v = C.c_void_p(), C.c_void_p()
        st = self._lib.tl_get_cache(self._h, int(seq_id), int(layer), C.byref(k), C.byref(v))
        if st != TL_OK:
            return None, None
        return k.value, v.value

    def get_cache_checked(self, seq_id: int, layer: int):
        k, v = C.c_void_p(), C.c_void_p()
        self._check(self._lib.tl_get_cache(self._h, int(seq_id), int(layer), C.byref(k), C.byref(v)))
        return k.value, v.value

    def append_kv(self, seq_id, layer, k_ptr, v_ptr, num_tokens, stream=0):
        self._check(self._lib.tl_append_kv(self._h, int(seq_id), int(layer), k_ptr, v_ptr,
                                           int(num_tokens), stream or None))

    def append_kv_all_layers(self, seq_ids, k_ptr, v_ptr, stream=0):
        self._check(self._lib.tl_append_kv_all_layers(self._h, _ids(seq_ids), len(seq_ids),
                                                      k_ptr, v_ptr, stream or None))

    def advance_seq_len(self, seq_id, num_tokens):
        self._check(self._lib.tl_advance_seq_len(self._h, int(seq_id), int(num_tokens)))

    def get_seq_len(self, seq_id) -> int:
        return self._lib.tl_get_seq_len(self._h, int(seq_id))

    def has_sequence(self, seq_id) -> bool:
        return bool(self._lib.tl_has_sequence(self._h, int(seq_id)))

    def used_memory(self) -> int:
        return self._lib.tl_used_memory(self._h)

    def total_memory(self) -> int:
        return self._lib.tl_total_memory(self._h)

    def free_memory(self) -> int:
        return self._lib.tl_free_memory(self._h)

    def active_sequence_count(self) -> int:
        return self._lib.tl_active_sequence_count(self._h)

    # -- paged / fused additions --------------------------------------------
    def block_table(self, seq_id):
        n = C.c_int(0)
        self._check(self._lib.tl_get_block_table(self._h, int(seq_id), None, 0, C.byref(n)))
        arr = (C.c_int * max(n.value, 1))()
        self._check(self._lib.tl_get_block_table(self._h, int(seq_id), arr, n.value, C.byref(n)))
        return list(arr[: n.value])

    def pool_stats(self) -> PoolStats:
        s = PoolStats()
        self._check(self._lib.tl_get_pool_stats(self._h, C.byref(s)))
        return s

    def pool(self):
        """(device base address, element count) of the pool [L][2][NB][block]."""
        base, n = C.c_void_p(), C.c_size_t()
        self._check(self._lib.tl_get_pool(self._h, C.byref(base), C.byref(n)))
        return base.value, n.value

    def permute_free_blocks(self, seed: int) -> None:
        self._check(self._lib.tl_permute_free_blocks(self._h, C.c_ulonglong(seed)))

    def decode_attention(self, layer, q_ptr, o_ptr, seq_ids, scale=0.0, stream=0):
        self._check(self._lib.tl_decode_attention(self._h, int(layer), q_ptr, o_ptr, _ids(seq_ids),
                                                  len(seq_ids), float(scale), stream or None))

    def attention_step(self, layer, q_ptr, k_ptr, v_ptr, o_ptr, seq_ids, scale=0.0, stream=0):
        """Appends one token per sequence in `layer`, then decodes (Q rotated
        like K when the cache rotates on append); advance afterwards."""
        self._check(self._lib.tl_attention_step(self._h, int(layer), q_ptr, k_ptr, v_ptr, o_ptr,
                                                _ids(seq_ids), len(seq_ids), float(scale),
                                                stream or None))

    def prefill_attention(self, layer, q_ptr, o_ptr, seq_ids, num_tokens, scale=0.0, stream=0):
        """Causal attention of each sequence's last num_tokens[i] written
        tokens (rows packed sequence after sequence in q/o)."""
        if len(num_tokens) != len(seq_ids):
            raise InvalidArgument(TL_ERR_INVALID_ARG, "seq_ids and num_tokens differ in length")
        self._check(self._lib.tl_prefill_attention(self._h, int(layer), q_ptr, o_ptr, _ids(seq_ids),
                                                   _ids(num_tokens), len(seq_ids), float(scale),
                                                   stream or None))

    def project_qkv_append(self, layer, x_ptr, hidden, wq, sq, wk, sk, wv, sv, group_size, seq_ids, q_ptr,
                           stream=0):
        """W8A16 Q/K/V projections of one decode token per sequence (x rows
        in seq_ids order); K and V are written at each sequence's current
        length, Q into q_ptr ([num_seqs][Hq*D])."""
        self._check(self._lib.tl_project_qkv_append(self._h, int(layer), x_ptr, int(hidden), wq, sq, wk, sk, wv,
                                                    sv, int(group_size), _ids(seq_ids), len(seq_ids), q_ptr,
                                                    stream or None))

    def project_qkv_append_packed(self, layer, x_ptr, hidden, wq, sq, wk, sk, wv, sv, group_size, seq_ids,
                                  q_ptr, stream=0):
        """project_qkv_append with wq/wk/wv repacked by pack_qkv_weight."""
        self._check(self._lib.tl_project_qkv_append_packed(self._h, int(layer), x_ptr, int(hidden), wq, sq, wk,
                                                           sk, wv, sv, int(group_size), _ids(seq_ids),
                                                           len(seq_ids), q_ptr, stream or None))

    # -- head-sharded peer gather (one process per GPU) ----------------------
    def peer_init(self, rank: int, world: int, gather_bytes: int) -> bytes:
        """Allocates this rank's gather region; returns its 64-byte IPC handle."""
        h = C.create_string_buffer(64)
        self._check(self._lib.tl_peer_init(self._h, int(rank), int(world), int(gather_bytes), h))
        return h.raw

    def peer_connect(self, handles: list[bytes]) -> None:
        blob = b"".join(handles)
        buf = C.create_string_buffer(blob, len(blob))
        self._check(self._lib.tl_peer_connect(self._h, buf))

    def peer_buffer(self):
        p, n = C.c_void_p(), C.c_size_t()
        self._check(self._lib.tl_peer_buffer(self._h, C.byref(p), C.byref(n)))
        return p.value, n.value

    def set_peer_wait_limit(self, seconds: float) -> None:
        """Limit of each wait for a peer's flag (<= 0: the built-in 10 s)."""
        self._check(self._lib.tl_set_peer_wait_limit(self._h, float(seconds)))

    def debug_peer_attach(self, rank: int, region_ptr: int) -> None:
        """Testing hook: a local device region stands in for rank `rank`'s
        IPC-shared peer region (one-GPU tests of the gather protocol)."""
        self._check(self._lib.tl_debug_peer_attach(self._h, int(rank), region_ptr))

    def decode_attention_peer(self, layer, q_ptr, seq_ids, out_offset, epoch, scale=0.0, stream=0):
        self._check(self._lib.tl_decode_attention_peer(self._h, int(layer), q_ptr, _ids(seq_ids),
                                                       len(seq_ids), float(scale), int(out_offset),
                                                       C.c_uint(epoch & 0xFFFFFFFF), stream or None))


    def sync_check(self, stream=0):
        self._check(self._lib.tl_sync_check(self._h, stream or None))


def rope_table(max_pos: int, head_dim: int, theta: float):
    """Host cos/sin tables [max_pos][D/2] (numpy float32), the handle's math."""
    import numpy as np
    lib = load()
    half = head_dim // 2
    cos = np.empty((max_pos, half), dtype=np.float32)
    sin = np.empty((max_pos, half), dtype=np.float32)
    fp = C.POINTER(C.c_float)
    lib.tl_rope_table(cos.ctypes.data_as(fp), sin.ctypes.data_as(fp), max_pos, head_dim, theta)
    return cos, sin


def decode_attention_static(view: PagedView, layer, q_ptr, o_ptr, table_rows, seq_lens,
                            scale=0.0, stream=0):
    """tl_decode_attention_static: decode over a caller-owned pool, with the
    library's file-scope split scratch (no allocation by the call)."""
    lib = load()
    buf = C.create_string_buffer(512)
    st = lib.tl_decode_attention_static(C.byref(view), int(layer), q_ptr, o_ptr, _ids(table_rows),
                                        _ids(seq_lens), len(seq_lens), float(scale),
                                        stream or None, buf, 512)
    if st != TL_OK:
        raise _ERRORS.get(st, TLError)(st, buf.value.decode())


def sample_tokens(logits_ptr, row_stride, rows, vocab, tokens_ptr, do_sample=False, temperature=1.0, top_k=50,
                  top_p=0.9, seed=0, step=0, stream=0):
    """tl_sample_tokens: one next token per row of fp16 logits, left in device
    memory (defaults as the reference's GenerationConfig: greedy unless
    do_sample; then top_p < 1, top_k > 0, or temperature)."""
    lib = load()
    st = lib.tl_sample_tokens(logits_ptr, int(row_stride), int(rows), int(vocab), int(bool(do_sample)),
                              float(temperature), int(top_k), float(top_p), int(seed) & (2**64 - 1),
                              int(step) & (2**64 - 1), tokens_ptr, stream or None)
    if st != TL_OK:
        raise _ERRORS.get(st, TLError)(st, lib.tl_last_error(None).decode())


def pack_qkv_weight(w_ptr, hidden, n, out_ptr, stream=0):
    """tl_qkv_pack_weight: int8 [hidden][n] weights into the tile-blocked
    layout project_qkv_append_packed reads (out: hidden * n bytes)."""
    lib = load()
    st = lib.tl_qkv_pack_weight(w_ptr, int(hidden), int(n), out_ptr, stream or None)
    if st != TL_OK:
        raise _ERRORS.get(st, TLError)(st, lib.tl_last_error(None).decode())


def inject_alloc_failure(nth: int) -> None:
    load().tl_debug_inject_alloc_failure(int(nth))

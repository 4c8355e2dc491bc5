"""ctypes loader for oracle/_ref/libtllm_ref.so: the reference's own
KVCacheManager and kernels::attention_decode compiled unmodified for sm_100a
(oracle/Makefile.ref). Test infrastructure: used as a checker only."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
REF_LIB = ROOT / "oracle" / "_ref" / "libtllm_ref.so"
_lib = None


def d2h(ptr: int, count: int):
    """Copies count fp16 values from a device address into a numpy uint16 array."""
    import numpy as np
    import torch  # noqa: F401  (loads libcudart.so.12)
    rt = C.CDLL("libcudart.so.12")
    rt.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    out = np.empty(count, dtype=np.uint16)
    assert rt.cudaMemcpy(out.ctypes.data, ptr, out.nbytes, 2) == 0
    return out


def available() -> bool:
    return REF_LIB.exists()


def load():
    global _lib
    if _lib is None:
        lib = C.CDLL(str(REF_LIB))
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        lib.ref_kv_create.argtypes = [i, i, i, i, i, C.POINTER(vp)]
        lib.ref_kv_allocate.argtypes = [vp, i, C.POINTER(i)]
        lib.ref_kv_append.argtypes = [vp, i, i, vp, vp, i, vp]
        lib.ref_kv_advance.argtypes = [vp, i, i]
        lib.ref_kv_get_cache.argtypes = [vp, i, i, C.POINTER(vp), C.POINTER(vp)]
        lib.ref_kv_destroy.argtypes = [vp]
        lib.ref_attention_decode.argtypes = [vp, vp, vp, vp, f, i, i, i, i, vp]
        lib.ref_attention_prefill.argtypes = [vp, vp, vp, vp, f, i, i, i, i, vp]
        lib.ref_w8a16_matmul.argtypes = [vp, vp, vp, vp, i, i, i, i, vp]
        lib.ref_last_error.restype = C.c_char_p
        _lib = lib
    return _lib


def attention_decode(q_dev, k_dev, v_dev, o_dev, scale, B, H, S, D):
    """kernels::attention_decode on [B][H][S][D] K/V (device pointers)."""
    rc = load().ref_attention_decode(q_dev, k_dev, v_dev, o_dev, scale, B, H, S, D, None)
    if rc != 0:
        raise RuntimeError("reference attention_decode failed: " + load().ref_last_error().decode())


def attention_prefill(q_dev, k_dev, v_dev, o_dev, scale, B, H, S, D):
    """kernels::attention_prefill on [B][H][S][D] Q/K/V/O (device pointers)."""
    rc = load().ref_attention_prefill(q_dev, k_dev, v_dev, o_dev, scale, B, H, S, D, None)
    if rc != 0:
        raise RuntimeError("reference attention_prefill failed: " + load().ref_last_error().decode())


class RefCache:
    """The reference KVCacheManager (contiguous slots)."""

    def __init__(self, L, H, D, max_seq_len, max_batch):
        self.lib = load()
        self.h = C.c_void_p()
        if self.lib.ref_kv_create(L, H, D, max_seq_len, max_batch, C.byref(self.h)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def allocate(self, max_len):
        sid = C.c_int()
        assert self.lib.ref_kv_allocate(self.h, max_len, C.byref(sid)) == 0
        return sid.value

    def append(self, sid, layer, k_dev, v_dev, n):
        rc = self.lib.ref_kv_append(self.h, sid, layer, k_dev, v_dev, n, None)
        if rc != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def advance(self, sid, n):
        assert self.lib.ref_kv_advance(self.h, sid, n) == 0

    def get_cache(self, sid, layer):
        k, v = C.c_void_p(), C.c_void_p()
        assert self.lib.ref_kv_get_cache(self.h, sid, layer, C.byref(k), C.byref(v)) == 0
        return k.value, v.value

    def close(self):
        if self.h:
            self.lib.ref_kv_destroy(self.h)
            self.h = None


def w8a16_matmul(x_dev, w_dev, s_dev, o_dev, M, N, K, group):
    """The reference's kernels::w8a16_matmul on device pointers (fp16 out)."""
    rc = load().ref_w8a16_matmul(x_dev, w_dev, s_dev, o_dev, M, N, K, group, None)
    if rc != 0:
        raise RuntimeError("reference w8a16_matmul failed: " + load().ref_last_error().decode())

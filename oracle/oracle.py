"""ctypes wrapper of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, always as the checker or
the timed CPU baseline, never as the product path. Every function documents
the reference code it restates in oracle.h.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
_lib = None


class PoolGeom(C.Structure):
    _fields_ = [("num_layers", C.c_int), ("num_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("block_size", C.c_int), ("num_blocks", C.c_int), ("head_major", C.c_int)]


def build() -> Path:
    src = [HERE / "oracle.c", HERE / "oracle.h", HERE / "Makefile"]
    if not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in src):
        subprocess.run(["make", "-C", str(HERE), "-s"], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        build()
        lib = C.CDLL(str(LIB))
        u16p, f32p, ip = C.POINTER(C.c_uint16), C.POINTER(C.c_float), C.POINTER(C.c_int)
        gp = C.POINTER(PoolGeom)
        lib.or_f32_to_f16.restype = C.c_uint16
        lib.or_f32_to_f16.argtypes = [C.c_float]
        lib.or_f16_to_f32.restype = C.c_float
        lib.or_f16_to_f32.argtypes = [C.c_uint16]
        lib.or_f32_to_f16_array.argtypes = [f32p, u16p, C.c_size_t]
        lib.or_f16_to_f32_array.argtypes = [u16p, f32p, C.c_size_t]
        lib.or_fill_normal_f16.argtypes = [u16p, C.c_size_t, C.c_uint64]
        lib.or_rope_table.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_float]
        lib.or_rope_row.argtypes = [u16p, u16p, C.c_int, C.c_int, f32p, f32p, C.c_int]
        lib.or_pool_offset.restype = C.c_size_t
        lib.or_pool_offset.argtypes = [gp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.or_append.argtypes = [u16p, gp, ip, C.c_int, C.c_int, C.c_int, u16p, u16p, f32p, f32p]
        lib.or_gather.argtypes = [u16p, gp, ip, C.c_int, C.c_int, u16p, u16p]
        lib.or_decode_one.argtypes = [u16p, u16p, u16p, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_float, C.c_double, f32p]
        lib.or_decode_paged_f32.restype = C.c_int
        lib.or_decode_paged_f32.argtypes = [u16p, gp, C.c_int, C.c_int, ip, C.c_int, ip, u16p,
                                            C.c_int, C.c_float, u16p, C.c_int]
        lib.or_w8a16_matmul.argtypes = [u16p, C.POINTER(C.c_int8), u16p, C.c_int, C.c_int, C.c_int,
                                        C.c_int, f32p, C.c_int]
        _lib = lib
    return _lib


def _u16(a):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_uint16))


def _f32(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _i32(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_int))


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    load().or_f32_to_f16_array(_f32(x), _u16(out), x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    load().or_f16_to_f32_array(_u16(h), _f32(out), h.size)
    return out


def normal_f16(shape, seed: int) -> np.ndarray:
    """Seeded N(0,1) fp16 bit patterns (splitmix64 + Box-Muller)."""
    out = np.empty(shape, dtype=np.uint16)
    load().or_fill_normal_f16(_u16(out), out.size, C.c_uint64(seed & (2**64 - 1)))
    return out


def rope_table(max_pos: int, head_dim: int, theta: float):
    half = head_dim // 2
    cos = np.empty((max_pos, half), dtype=np.float32)
    sin = np.empty((max_pos, half), dtype=np.float32)
    load().or_rope_table(_f32(cos), _f32(sin), max_pos, head_dim, theta)
    return cos, sin


def rope_row(row: np.ndarray, cos, sin, pos: int) -> np.ndarray:
    """row: uint16 [Hkv][D] -> rotated copy."""
    row = np.ascontiguousarray(row, dtype=np.uint16)
    out = np.empty_like(row)
    H, D = row.shape
    load().or_rope_row(_u16(out), _u16(row), H, D, _f32(cos), _f32(sin), pos)
    return out


def geom(num_layers, num_kv_heads, head_dim, block_size, num_blocks, head_major=False):
    return PoolGeom(num_layers, num_kv_heads, head_dim, block_size, num_blocks, int(head_major))


def pool_offset(g: PoolGeom, layer, kv, block, tok, head) -> int:
    return load().or_pool_offset(C.byref(g), layer, kv, block, tok, head)


def append(pool: np.ndarray, g: PoolGeom, bt: np.ndarray, layer: int, pos0: int, k: np.ndarray,
           v: np.ndarray, cos=None, sin=None) -> None:
    """In-place paged append of rows k/v [n][Hkv][D] at positions pos0.."""
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    bt = np.ascontiguousarray(bt, dtype=np.int32)
    n = k.shape[0]
    load().or_append(_u16(pool), C.byref(g), _i32(bt), layer, pos0, n, _u16(k), _u16(v),
                     _f32(cos) if cos is not None else None, _f32(sin) if sin is not None else None)


def gather(pool: np.ndarray, g: PoolGeom, bt: np.ndarray, layer: int, S: int):
    bt = np.ascontiguousarray(bt, dtype=np.int32)
    k = np.empty((S, g.num_kv_heads, g.head_dim), dtype=np.uint16)
    v = np.empty_like(k)
    if S:
        load().or_gather(_u16(pool), C.byref(g), _i32(bt), layer, S, _u16(k), _u16(v))
    return k, v


def decode_one(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, eps: float = 0.0):
    """fp64 GQA decode for one sequence: q [Hq][D], k/v [S][Hkv][D] (uint16)."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    Hq, D = q.shape
    S = k.shape[0]
    Hkv = k.shape[1] if S else Hq
    out = np.empty((Hq, D), dtype=np.float32)
    load().or_decode_one(_u16(q), _u16(k) if S else None, _u16(v) if S else None, S, Hq, Hkv, D,
                         scale, eps, _f32(out))
    return out


def decode_paged_f32(pool, g: PoolGeom, layer, bt: np.ndarray, lens: np.ndarray, q: np.ndarray,
                     num_q_heads: int, scale: float, threads: int = 0):
    """The timed fp32 CPU baseline over a host copy of the paged pool."""
    bt = np.ascontiguousarray(bt, dtype=np.int32)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    q = np.ascontiguousarray(q, dtype=np.uint16)
    out = np.empty_like(q)
    used = load().or_decode_paged_f32(_u16(pool), C.byref(g), layer, len(lens), _i32(bt),
                                      bt.shape[1], _i32(lens), _u16(q), num_q_heads, scale,
                                      _u16(out), threads)
    return out, used


def w8a16_matmul(x: np.ndarray, w: np.ndarray, scales: np.ndarray, group: int, threads: int = 0) -> np.ndarray:
    """The reference's W8A16 projection in fp32 (its exact operation order):
    x [M][K] fp16 bits (uint16), w [K][N] int8, scales [K/group][N] fp16 bits.
    Returns fp32 [M][N]; the reference's output is that rounded to fp16."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    M, K = x.shape
    N = w.shape[1]
    assert w.shape[0] == K and scales.shape == ((K + group - 1) // group, N)
    out = np.empty((M, N), dtype=np.float32)
    load().or_w8a16_matmul(_u16(x), w.ctypes.data_as(C.POINTER(C.c_int8)), _u16(scales), M, N, K, group,
                           _f32(out), threads or (os.cpu_count() or 1))
    return out

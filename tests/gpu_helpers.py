"""GPU-side helpers for the parity tests: device buffers (torch), raw copies
of library-owned memory, and a driver that runs the paged path and the CPU
oracle side by side on the same seeded inputs."""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

import numpy as np

import oracle as O
import tiny_llm_b200 as T

ATOL, RTOL = 2e-3, 1e-3  # attention tolerance: |got - ref| <= ATOL + RTOL*|ref|

_cudart = None


def cudart():
    """The CUDA runtime torch already loaded (same primary context)."""
    global _cudart
    if _cudart is None:
        import torch  # noqa: F401  (loads libcudart.so.12)
        _cudart = C.CDLL("libcudart.so.12")
        _cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
        _cudart.cudaMemcpy.restype = C.c_int
    return _cudart


def d2h(ptr: int, count: int, dtype=np.uint16) -> np.ndarray:
    out = np.empty(count, dtype=dtype)
    rc = cudart().cudaMemcpy(out.ctypes.data, ptr, out.nbytes, 2)
    assert rc == 0, f"cudaMemcpy D2H failed: {rc}"
    return out


def to_dev(a: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def from_dev(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def check_close(got: np.ndarray, ref: np.ndarray, what: str = "") -> tuple[float, float]:
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    bound = ATOL + RTOL * np.abs(ref.astype(np.float64))
    bad = err > bound
    max_abs = float(err.max()) if err.size else 0.0
    rel = err / np.maximum(np.abs(ref.astype(np.float64)), 1e-6)
    max_rel = float(rel[np.abs(ref) > 1e-2].max()) if np.any(np.abs(ref) > 1e-2) else 0.0
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} outside tolerance; "
                           f"max_abs={max_abs:.3e} max_rel={max_rel:.3e}")
    return max_abs, max_rel


@dataclass
class Run:
    """A cache plus the oracle's logical copy of every sequence's K/V."""
    cache: T.KVCache
    L: int
    Hq: int
    Hkv: int
    D: int
    bs: int
    rope: bool
    theta: float
    seqs: list = field(default_factory=list)
    logical_k: dict = field(default_factory=dict)  # (sid, layer) -> list of rows [Hkv][D]
    logical_v: dict = field(default_factory=dict)
    cos: np.ndarray | None = None
    sin: np.ndarray | None = None

    @classmethod
    def create(cls, L, Hq, Hkv, D, bs, max_seq_len, max_batch, rope=False, theta=10000.0,
               layout=T.TL_LAYOUT_TOKEN_MAJOR, num_blocks=0, permute_seed=None):
        cache = T.KVCache(num_layers=L, num_kv_heads=Hkv, head_dim=D, max_seq_len=max_seq_len,
                          max_batch_size=max_batch, block_size=bs, num_blocks=num_blocks,
                          num_q_heads=Hq, rope_theta=theta, rope_on_append=rope, layout=layout)
        if permute_seed is not None:
            cache.permute_free_blocks(permute_seed)
        r = cls(cache, L, Hq, Hkv, D, bs, rope, theta)
        if rope:
            r.cos, r.sin = O.rope_table(max_seq_len, D, theta)
        return r

    def allocate(self, max_len) -> int:
        sid = self.cache.allocate_sequence(max_len)
        self.seqs.append(sid)
        for l in range(self.L):
            self.logical_k[(sid, l)] = []
            self.logical_v[(sid, l)] = []
        return sid

    def _record(self, sid, layer, pos0, k, v):
        for j in range(k.shape[0]):
            row = k[j]
            if self.rope:
                row = O.rope_row(row, self.cos, self.sin, pos0 + j)
            lk, lv = self.logical_k[(sid, layer)], self.logical_v[(sid, layer)]
            p = pos0 + j
            if p < len(lk):  # overwrite (same position appended again)
                lk[p], lv[p] = row, v[j]
            else:
                assert p == len(lk)
                lk.append(row)
                lv.append(v[j].copy())

    def prefill(self, sid, P, seed):
        """Per-layer multi-token append (reference appendKV path), then advance."""
        pos0 = self.cache.get_seq_len(sid)
        for l in range(self.L):
            k = O.normal_f16((P, self.Hkv, self.D), seed * 1000 + 2 * l)
            v = O.normal_f16((P, self.Hkv, self.D), seed * 1000 + 2 * l + 1)
            kd, vd = to_dev(k), to_dev(v)
            self.cache.append_kv(sid, l, kd.data_ptr(), vd.data_ptr(), P)
            self._record(sid, l, pos0, k, v)
        self.cache.advance_seq_len(sid, P)

    def step_append(self, sids, seed):
        """Fused all-layer append of one token per sequence."""
        B = len(sids)
        k = O.normal_f16((self.L, B, self.Hkv, self.D), seed)
        v = O.normal_f16((self.L, B, self.Hkv, self.D), seed + 1)
        kd, vd = to_dev(k), to_dev(v)
        self.cache.append_kv_all_layers(sids, kd.data_ptr(), vd.data_ptr())
        for i, sid in enumerate(sids):
            pos = self.cache.get_seq_len(sid)
            for l in range(self.L):
                self._record(sid, l, pos, k[l, i:i + 1], v[l, i:i + 1])
        return kd, vd

    def decode_and_check(self, layer, sids, seed, scale=None):
        import torch
        B = len(sids)
        q = O.normal_f16((B, self.Hq, self.D), seed)
        qd = to_dev(q)
        od = torch.full((B, self.Hq, self.D), 0x7e00, dtype=torch.int16, device="cuda")  # NaN fill
        sc = scale if scale is not None else 1.0 / math.sqrt(self.D)
        self.cache.decode_attention(layer, qd.data_ptr(), od.data_ptr(), sids, sc)
        self.cache.sync_check()
        got = O.f16_to_f32(from_dev(od))
        worst = (0.0, 0.0)
        for i, sid in enumerate(sids):
            lk = self.logical_k[(sid, layer)]
            S = len(lk)
            k = np.stack(lk) if S else np.zeros((0, self.Hkv, self.D), np.uint16)
            v = np.stack(self.logical_v[(sid, layer)]) if S else k
            ref = O.decode_one(q[i], k, v, sc)
            ma, mr = check_close(got[i], ref, f"layer {layer} seq {sid} S={S}")
            worst = (max(worst[0], ma), max(worst[1], mr))
        return worst

    def attention_step_and_check(self, layer, sids, seed, scale=None):
        """tl_attention_step for one layer: appends one new token per
        sequence, decodes with Q rotated like K, and checks the output
        against the oracle (RoPE row on Q at the new token's position, fp64
        attention over every token including the new one)."""
        import torch
        B = len(sids)
        k = O.normal_f16((B, self.Hkv, self.D), seed)
        v = O.normal_f16((B, self.Hkv, self.D), seed + 1)
        q = O.normal_f16((B, self.Hq, self.D), seed + 2)
        kd, vd, qd = to_dev(k), to_dev(v), to_dev(q)
        od = torch.full((B, self.Hq, self.D), 0x7e00, dtype=torch.int16, device="cuda")  # NaN fill
        sc = scale if scale is not None else 1.0 / math.sqrt(self.D)
        self.cache.attention_step(layer, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(),
                                  sids, sc)
        self.cache.sync_check()
        got = O.f16_to_f32(from_dev(od))
        for i, sid in enumerate(sids):
            pos = self.cache.get_seq_len(sid)
            self._record(sid, layer, pos, k[i:i + 1], v[i:i + 1])
            qi = O.rope_row(q[i], self.cos, self.sin, pos) if self.rope else q[i]
            kk = np.stack(self.logical_k[(sid, layer)])
            vv = np.stack(self.logical_v[(sid, layer)])
            ref = O.decode_one(qi, kk, vv, sc)
            check_close(got[i], ref, f"attention step layer {layer} seq {sid} pos {pos}")

    def check_pool_bit_exact(self):
        """Gathers every sequence back from the device pool via its block
        table and compares bit-for-bit with the oracle's logical K/V."""
        base, n = self.cache.pool()
        pool = d2h(base, n)
        nb = self.cache.config.num_blocks
        g = O.geom(self.L, self.Hkv, self.D, self.bs, nb,
                   self.cache.config.layout == T.TL_LAYOUT_HEAD_MAJOR)
        for sid in self.seqs:
            bt = np.array(self.cache.block_table(sid), np.int32)
            for l in range(self.L):
                lk = self.logical_k[(sid, l)]
                S = len(lk)
                if S == 0:
                    continue
                k, v = O.gather(pool, g, bt, l, S)
                assert np.array_equal(k, np.stack(lk)), f"K mismatch seq {sid} layer {l}"
                assert np.array_equal(v, np.stack(self.logical_v[(sid, l)])), f"V mismatch seq {sid} layer {l}"

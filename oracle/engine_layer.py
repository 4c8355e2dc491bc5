"""CPU restatement of tiny-llm's decoder layer, for the engine drop-in tests.

TEST INFRASTRUCTURE ONLY: the checker of tests/test_gpu_engine.py, never used
by the product. Restates, per token row:

* TransformerLayer::forward / forwardPrefill (reference
  src/transformer.cpp:123-198): x += attention(rmsnorm(x, rms_att));
  x += ffn(rmsnorm(x, rms_ffn));
* attention (src/transformer.cpp:200-248) with the paged path's meaning:
  Q/K/V projections, the new K/V rows appended to the sequence's cache, each
  row attending the cached tokens up to its own position with query head h
  reading KV head h // (Hq / Hkv) (the oracle's fp64 decode_one), then the
  output projection;
* feedForward (src/transformer.cpp:250-276): SwiGLU, w2(silu(w1 x) * w3 x);
* rmsnorm (kernels/rmsnorm.cu:10-60): x / sqrt(mean(x^2) + eps) * w, in
  float64 here (the kernel sums in fp32);
* add_inplace and silu_mul_inplace (kernels/elementwise.cu:7-25);
* every W8A16 projection with oracle.w8a16_matmul, which equals the
  reference's kernels::w8a16_matmul bit for bit.
Every intermediate the reference stores as fp16 is rounded to fp16 here at
the same point.
"""
from __future__ import annotations

import math

import numpy as np

import oracle as O


def _v(h: np.ndarray) -> np.ndarray:
    return O.f16_to_f32(h).astype(np.float64)


def _h(x: np.ndarray) -> np.ndarray:
    return O.f32_to_f16(np.asarray(x, dtype=np.float32))


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    xv = _v(x)
    r = 1.0 / np.sqrt((xv * xv).mean(axis=-1, keepdims=True) + eps)
    return _h(xv * r * _v(w))


class Layer:
    """One decoder layer with its own KV cache rows (logical, per sequence)."""

    def __init__(self, weights: dict, hidden: int, heads: int, kv_heads: int, head_dim: int,
                 inter: int, group: int, eps: float = 1e-5):
        self.w = weights
        self.hidden, self.Hq, self.Hkv, self.D = hidden, heads, kv_heads, head_dim
        self.inter, self.group, self.eps = inter, group, eps
        self.k: dict[int, list] = {}
        self.v: dict[int, list] = {}

    def _proj(self, x: np.ndarray, name: str, rows: int, cols: int) -> np.ndarray:
        w = self.w[name + ".w"].view(np.int8).reshape(rows, cols)
        s = self.w[name + ".s"].reshape(-1, cols)
        return _h(O.w8a16_matmul(x, w, s, self.group))

    def step(self, seq: int, x: np.ndarray) -> np.ndarray:
        """Rows x [T][hidden] (fp16 bits) at the sequence's next T positions:
        forwardPrefill when T > 1, forward when T == 1. Returns the new x."""
        H, Hq, Hkv, D, F = self.hidden, self.Hq, self.Hkv, self.D, self.inter
        T = x.shape[0]
        n = rmsnorm(x, self.w["rms_att"], self.eps)
        q = self._proj(n, "wq", H, Hq * D).reshape(T, Hq, D)
        k = self._proj(n, "wk", H, Hkv * D).reshape(T, Hkv, D)
        v = self._proj(n, "wv", H, Hkv * D).reshape(T, Hkv, D)
        ks, vs = self.k.setdefault(seq, []), self.v.setdefault(seq, [])
        pos0 = len(ks)
        ks.extend(k)
        vs.extend(v)
        kk, vv = np.stack(ks), np.stack(vs)
        scale = 1.0 / math.sqrt(D)
        attn = np.stack([_h(O.decode_one(q[t], kk[:pos0 + t + 1], vv[:pos0 + t + 1], scale))
                         for t in range(T)]).reshape(T, Hq * D)
        o = self._proj(attn, "wo", Hq * D, H)
        x = _h(_v(x) + _v(o))
        n2 = rmsnorm(x, self.w["rms_ffn"], self.eps)
        g = _v(self._proj(n2, "w1", H, F))
        u = _v(self._proj(n2, "w3", H, F))
        hmid = _h((g / (1.0 + np.exp(-g))) * u)
        f = self._proj(hmid, "w2", F, H)
        return _h(_v(x) + _v(f))


class Model:
    """The whole model of InferenceEngine::generate (reference
    src/inference_engine.cpp:113-294) with greedy sampling: embedding gather
    (kernels/elementwise.cu:27-43), every layer's forwardPrefill over the
    prompt, then per token the final RMSNorm, the LM-head projection to fp16
    logits and sampleGreedy's first largest logit (:346-362), fed back
    through every layer's forward."""

    def __init__(self, dump: dict, layers: int, hidden: int, heads: int, kv_heads: int, head_dim: int,
                 inter: int, vocab: int, group: int, eps: float = 1e-5):
        self.layers = []
        for l in range(layers):
            p = f"L{l}."
            w = {k[len(p):]: v for k, v in dump.items() if k.startswith(p)}
            self.layers.append(Layer(w, hidden, heads, kv_heads, head_dim, inter, group, eps))
        self.emb = dump["embedding"].reshape(vocab, hidden)
        self.norm = dump["final_norm"]
        self.head_w = dump["lm_head.w"].view(np.int8).reshape(hidden, vocab)
        self.head_s = dump["lm_head.s"].reshape(-1, vocab)
        self.group, self.eps = group, eps

    def _forward(self, rows: np.ndarray) -> np.ndarray:
        for lay in self.layers:
            rows = lay.step(0, rows)
        return rows

    def _next(self, row: np.ndarray):
        logits = O.f16_to_f32(_h(O.w8a16_matmul(rmsnorm(row, self.norm, self.eps), self.head_w, self.head_s,
                                                self.group)))[0].astype(np.float64)
        t = int(np.argmax(logits))  # the first index of the largest
        rest = np.delete(logits, t)
        return t, float(logits[t] - rest.max()) if rest.size else np.inf

    def generate(self, prompt: list[int], max_new: int):
        """(greedy tokens, per token the gap between the largest and the
        second-largest logit)."""
        x = self._forward(self.emb[np.asarray(prompt)])
        tokens, gaps = [], []
        for i in range(max_new):
            t, gap = self._next(x[-1:])
            tokens.append(t)
            gaps.append(gap)
            if i + 1 < max_new:
                x = self._forward(self.emb[[t]])
        return tokens, gaps


def read_dump(path) -> dict:
    """Arrays written by oracle/engine/engine_harness.cpp (its Dump format)."""
    kinds = {b"h": np.uint16, b"b": np.uint8, b"i": np.int32}
    out = {}
    with open(path, "rb") as f:
        while True:
            head = f.read(4)
            if not head:
                break
            n = int.from_bytes(head, "little")
            name = f.read(n).decode()
            kind = f.read(1)
            count = int.from_bytes(f.read(8), "little")
            dt = np.dtype(kinds[kind])
            out[name] = np.frombuffer(f.read(count * dt.itemsize), dtype=dt).copy()
    return out

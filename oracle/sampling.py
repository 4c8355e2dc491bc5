"""CPU restatement of the reference's next-token samplers.

TEST INFRASTRUCTURE ONLY: the checker for tests/ and bench.py's cpu_baseline
leg; never used by the product. Restates InferenceEngine::sample and its
strategies (reference src/inference_engine.cpp:330-490) in float64:

* greedy: the first index of the largest logit (:346-362; a NaN first logit
  is returned, other NaNs never win, -0 equals +0);
* temperature (:365-397), top-k (:400-436), top-p (:439-489), with the
  reference's clamps (T >= 1e-5, k in [1, V], p in [1e-5, 1]) and its
  precedence (do_sample, then top_p < 1, then top_k > 0, then temperature);
* candidates in descending logit order, equal logits by ascending index (the
  reference's std::sort / std::partial_sort leave that order unspecified);
* the draw: an inverse CDF over the candidates in that order at the uniform
  u of (seed, step, row) that the device sampler uses (splitmix64, 24 bits);
  the reference draws with std::mt19937 + std::discrete_distribution, i.e.
  the same distribution with other random numbers.
NaN logits weigh 0 in the stochastic strategies (the reference's sums turn
NaN).
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1


def uniform(seed: int, step: int, row: int) -> float:
    """The device sampler's uniform in [0, 1): splitmix64 of (seed, step, row)."""
    z = (seed ^ ((0x9E3779B97F4A7C15 * (row + 1)) & M64) ^ ((0xD1B54A32D192ED03 * (step + 1)) & M64)) & M64
    z = (z + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    z ^= z >> 31
    return float(np.float32((z >> 40) * (1.0 / 16777216.0)))


def mode_of(do_sample: bool, top_k: int, top_p: float) -> str:
    if not do_sample:
        return "greedy"
    if top_p < 1.0:
        return "top_p"
    if top_k > 0:
        return "top_k"
    return "temperature"


def greedy(logits: np.ndarray) -> int:
    """logits: float values (NaN allowed) of one row."""
    x = np.asarray(logits, dtype=np.float64)
    if x.size == 0:
        return 0
    best, bi = x[0], 0
    for i in range(1, x.size):  # sampleGreedy's loop: `>` never holds for NaN
        if x[i] > best:
            best, bi = x[i], i
    return bi


def candidates(logits: np.ndarray, do_sample=True, temperature=1.0, top_k=50, top_p=0.9):
    """(indices in draw order, their weights exp((l - max) / T), mode)."""
    x = np.asarray(logits, dtype=np.float64)
    V = x.size
    mode = mode_of(do_sample, top_k, top_p)
    T = max(float(np.float32(temperature)), 1e-5)
    valid = ~np.isnan(x)
    order = np.lexsort((np.arange(V), -np.where(valid, x, -np.inf)))  # value desc, index asc
    m = np.max(x[valid]) if valid.any() else 0.0
    w = np.where(valid, np.exp((np.where(valid, x, m) - m) / T), 0.0)
    if mode == "top_k":
        k = max(1, min(int(top_k), V))
        idx = order[:k]
    elif mode == "top_p":
        p = min(max(float(np.float32(top_p)), 1e-5), 1.0)
        ws = w[order]
        cum = np.cumsum(ws) / ws.sum()
        cut = int(np.searchsorted(cum, p, side="left")) + 1  # first i with cumsum >= p
        idx = order[:min(cut, V)]
    else:
        idx = order
    return idx, w[idx], mode


def sample(logits, do_sample=False, temperature=1.0, top_k=50, top_p=0.9, seed=0, step=0, row=0):
    """(token, margin): margin = distance of the draw (and, for top-p, of the
    cutoff) from the nearest boundary, as a fraction of the total weight;
    draws closer than ~1e-4 may differ between float32 and float64 sums."""
    x = np.asarray(logits, dtype=np.float64)
    if mode_of(do_sample, top_k, top_p) == "greedy" or x.size == 0:
        return greedy(x), 1.0
    idx, w, mode = candidates(x, do_sample, temperature, top_k, top_p)
    total = w.sum()
    if not total > 0:
        return greedy(x), 1.0
    u = uniform(seed, step, row)
    cum = np.cumsum(w)
    target = u * total
    j = int(np.searchsorted(cum, target, side="right"))
    j = min(j, len(idx) - 1)
    bounds = np.concatenate(([0.0], cum))
    margin = float(np.min(np.abs(bounds - target)) / total)
    if mode == "top_p":
        allw = np.where(np.isnan(x), 0.0, np.exp((np.where(np.isnan(x), 0, x) - np.nanmax(x)) /
                                                   max(float(np.float32(temperature)), 1e-5)))
        ordw = np.sort(allw)[::-1]
        c = np.cumsum(ordw) / ordw.sum()
        p = min(max(float(np.float32(top_p)), 1e-5), 1.0)
        margin = min(margin, float(np.min(np.abs(c - p))))
    return int(idx[j]), margin


def window(logits, do_sample=True, temperature=1.0, top_k=50, top_p=0.9, seed=0, step=0, row=0, tol=1e-4):
    """The tokens a float32 implementation of the same draw may return: those
    whose CDF interval meets [target - tol, target + tol] (as fractions of
    the total), over the oracle's candidate set and, for top-p, the cutoffs
    up to two tokens either side of it whose cumulative mass is within tol
    of p."""
    x = np.asarray(logits, dtype=np.float64)
    if mode_of(do_sample, top_k, top_p) == "greedy" or x.size == 0:
        return {greedy(x)}
    idx, w, mode = candidates(x, do_sample, temperature, top_k, top_p)
    sets = [(idx, w)]
    if mode == "top_p":
        valid = ~np.isnan(x)
        T = max(float(np.float32(temperature)), 1e-5)
        m = np.max(x[valid])
        allw = np.where(valid, np.exp((np.where(valid, x, m) - m) / T), 0.0)
        order = np.lexsort((np.arange(x.size), -np.where(valid, x, -np.inf)))
        c = np.cumsum(allw[order]) / allw.sum()
        p = min(max(float(np.float32(top_p)), 1e-5), 1.0)
        cut = len(idx)
        for n in range(max(1, cut - 2), min(cut + 2, x.size) + 1):  # cutoffs float32 sums could pick
            if n != cut and abs(c[n - 1] - p) < tol:
                sets.append((order[:n], allw[order[:n]]))
    u = uniform(seed, step, row)
    out = set()
    for ids, ws in sets:
        total = ws.sum()
        if not total > 0:
            continue
        cum = np.concatenate(([0.0], np.cumsum(ws))) / total
        hit = (cum[1:] > u - tol) & (cum[:-1] <= u + tol)
        out.update(int(i) for i in np.asarray(ids)[hit])
    return out

"""tl_sample_tokens on the device vs the oracle's restatement of the
reference's samplers: greedy bit for bit; the stochastic strategies token
for token at the same uniform, up to the tokens whose CDF steps lie within
1e-4 of the draw (where float32 and float64 sums may part), and in
distribution over many rows."""
import sys
from pathlib import Path

import numpy as np
import pytest

import conftest
import oracle as O
import tiny_llm_b200 as T
from gpu_helpers import to_dev

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
import sampling as S  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_gpu():
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")


def _run(lg, rows, V, stride, **kw):
    import torch
    ld = to_dev(lg)
    td = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    T.sample_tokens(ld.data_ptr(), stride, rows, V, td.data_ptr(), **kw)
    torch.cuda.synchronize()
    return td.cpu().numpy()


@pytest.mark.parametrize("V", [1, 7, 1000, 32000, 128256])
def test_greedy_bit_exact(V):
    rows = 16
    rng = np.random.default_rng(V)
    x = np.round(rng.normal(0, 3, (rows, V)) * 4) / 4  # coarse: many ties
    lg = O.f32_to_f16(x.astype(np.float32))
    if V > 3:
        lg[1, :] = 0x8000  # all -0 ...
        lg[1, 3] = 0x0000  # ... and one +0: equal, the first wins
        lg[2, 0] = 0x7E00  # NaN first: index 0 (the reference's loop)
        lg[3, 5] = 0x7E00  # NaN elsewhere: never wins
        lg[4, :] = 0x7E00  # all NaN: 0
    got = _run(lg, rows, V, V)
    exp = [S.greedy(O.f16_to_f32(lg[r]).astype(np.float64)) for r in range(rows)]
    assert list(got) == exp


@pytest.mark.parametrize("V", [7, 1000, 32000])
@pytest.mark.parametrize("kw", [
    dict(temperature=0.7, top_k=0, top_p=1.0),
    dict(temperature=1.0, top_k=50, top_p=1.0),
    dict(temperature=1.3, top_k=1, top_p=1.0),
    dict(temperature=1.0, top_k=1000000, top_p=1.0),
    dict(temperature=0.8, top_k=50, top_p=0.9),
    dict(temperature=1.0, top_k=0, top_p=0.999),
    dict(temperature=1.0, top_k=0, top_p=-1.0),
    dict(temperature=1e-8, top_k=0, top_p=1.0),
])
def test_draws_match_oracle(V, kw):
    rows = 128
    rng = np.random.default_rng(V + int(kw["temperature"] * 10))
    x = np.round(rng.normal(0, 3, (rows, V)) * 8) / 8
    lg = O.f32_to_f16(x.astype(np.float32))
    seed, step = 1234 + V, 7
    got = _run(lg, rows, V, V, do_sample=True, seed=seed, step=step, **kw)
    sharp = 0
    for r in range(rows):
        xr = O.f16_to_f32(lg[r]).astype(np.float64)
        ok = S.window(xr, True, seed=seed, step=step, row=r, tol=1e-4, **kw)
        assert int(got[r]) in ok, f"row {r}: {got[r]} not in {sorted(ok)[:8]}"
        sharp += len(ok) == 1
    # the check is one token exactly for most rows (fewer when thousands of
    # tokens share the mass and their CDF steps are narrower than 1e-4)
    assert sharp >= rows // 4


def test_distribution_over_rows():
    """8192 rows sharing one row of logits (row_stride 0), temperature 1:
    every token's frequency within 5 standard deviations of its probability."""
    rows, V = 8192, 40
    x = np.random.default_rng(3).normal(0, 1.5, V).astype(np.float32)
    lg = O.f32_to_f16(x)[None, :]
    got = _run(lg, rows, V, 0, do_sample=True, temperature=1.0, top_k=0, top_p=1.0, seed=99, step=1)
    xv = O.f16_to_f32(lg[0]).astype(np.float64)
    p = np.exp(xv - xv.max())
    p /= p.sum()
    f = np.bincount(got, minlength=V) / rows
    assert np.all(np.abs(f - p) <= 5 * np.sqrt(p * (1 - p) / rows) + 1e-3)


@pytest.mark.parametrize("kw", [
    dict(temperature=0.5, top_k=1000, top_p=1.0),    # the k-th largest inside 5000 ties
    dict(temperature=0.01, top_k=0, top_p=0.5),      # 3000 tied maxima, half the mass
    dict(temperature=0.02, top_k=0, top_p=0.97),     # cutoff inside the second tie group
])
def test_draws_with_many_ties_at_the_cutoff(kw):
    """Thousands of equal logits at the candidate cutoff under low
    temperature: the drawn index among the ties (ascending) must be the
    oracle's, never the pre-set argmax standing in for it."""
    rows, V = 64, 32000
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (rows, V)).astype(np.float32) - 8.0
    if kw["top_k"]:
        x[:, rng.choice(V, 10, replace=False)] = 5.0
        x[:, rng.choice(V, 5000, replace=False)] = 4.75
    else:
        top = rng.choice(V, 6000, replace=False)
        x[:, top[:3000]] = 5.0
        x[:, top[3000:]] = 4.96875
    lg = O.f32_to_f16(x)
    seed, step = 77, 3
    got = _run(lg, rows, V, V, do_sample=True, seed=seed, step=step, **kw)
    argmax_hits = 0
    for r in range(rows):
        xr = O.f16_to_f32(lg[r]).astype(np.float64)
        ok = S.window(xr, True, seed=seed, step=step, row=r, tol=1e-4, **kw)
        assert int(got[r]) in ok, f"row {r}: {got[r]} not in {sorted(ok)[:8]}"
        argmax_hits += int(got[r]) == S.greedy(xr)
    assert argmax_hits < rows // 2


@pytest.mark.parametrize("V", [65537, 524287, 524288])
def test_largest_vocabularies(V):
    """Rows split over the cluster's 8 slices just past one slice (65537)
    and at the largest supported vocabulary (8 x 65536): greedy bit for bit
    (the maximum placed in the first and in the last key), and top-k/top-p
    draws at the oracle's uniform."""
    rows = 6
    rng = np.random.default_rng(V)
    x = np.round(rng.normal(0, 3, (rows, V)) * 8) / 8
    x[0, V - 1] = 40.0
    x[1, 0] = 40.0
    lg = O.f32_to_f16(x.astype(np.float32))
    got = _run(lg, rows, V, V)
    exp = [S.greedy(O.f16_to_f32(lg[r]).astype(np.float64)) for r in range(rows)]
    assert list(got) == exp
    assert exp[0] == V - 1 and exp[1] == 0
    kw = dict(temperature=0.8, top_k=50, top_p=0.9)
    seed, step = 77, 3
    got = _run(lg, rows, V, V, do_sample=True, seed=seed, step=step, **kw)
    for r in range(rows):
        xr = O.f16_to_f32(lg[r]).astype(np.float64)
        ok = S.window(xr, True, seed=seed, step=step, row=r, tol=1e-4, **kw)
        assert int(got[r]) in ok, f"row {r}: {got[r]} not in {sorted(ok)[:8]}"

"""Next-token sampling: the oracle's restatement of the reference's samplers
(src/inference_engine.cpp:330-490) on the reference's own test cases
(tests/test_inference_engine.cu:61-256), and tl_sample_tokens' argument
checks (no device needed)."""
import sys
from pathlib import Path

import numpy as np
import pytest

import tiny_llm_b200 as T

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "oracle"))
import sampling as S  # noqa: E402


def logits(n, scale, seed):
    return np.random.default_rng(seed).normal(0.0, scale, n).astype(np.float16).astype(np.float64)


def test_greedy_is_first_argmax():  # :61-82
    x = logits(1000, 10.0, 123)
    assert S.greedy(x) == int(np.argmax(x))
    y = np.zeros(100)
    y[42] = 100.0
    assert S.greedy(y) == 42
    assert S.greedy(np.array([1.0])) == 0  # :177-180
    z = np.array([0.0, 3.0, 1.0, 3.0])
    assert S.greedy(z) == 1  # ties: the first
    assert S.greedy(np.array([-0.0, 0.0])) == 0  # -0 == +0
    assert S.greedy(np.array([np.nan, 5.0])) == 0 and S.greedy(np.array([1.0, np.nan, 5.0])) == 2


@pytest.mark.parametrize("kw", [dict(top_k=0, top_p=1.0), dict(top_k=50, top_p=1.0), dict(top_k=0, top_p=0.9)])
def test_draws_are_valid_indices(kw):  # :84-118
    x = logits(1000, 10.0, 456)
    for i in range(100):
        t, _ = S.sample(x, True, 1.0, seed=i, **kw)
        assert 0 <= t < 1000


def test_low_temperature_approaches_greedy():  # :120-136
    x = logits(100, 10.0, 202)
    g = S.greedy(x)
    assert sum(S.sample(x, True, 0.01, top_k=0, top_p=1.0, seed=i)[0] == g for i in range(100)) >= 95


def test_clamps():  # :138-256
    x = logits(8, 10.0, 404)
    assert 0 <= S.sample(x, True, 1.0, top_k=64, top_p=1.0, seed=11)[0] < 8  # k > V
    assert 0 <= S.sample(x, True, 1.0, top_k=0, top_p=1.0, seed=23)[0] < 8  # k <= 0: temperature
    assert 0 <= S.sample(x, True, 0.0, top_k=0, top_p=1.0, seed=19)[0] < 8  # T <= 0 -> 1e-5
    # p <= tiny: only the largest logit remains
    assert S.sample(x, True, 1.0, top_k=0, top_p=-1.0, seed=13)[0] == S.greedy(x)
    assert S.sample(x, True, 1.0, top_k=0, top_p=1e-8, seed=29)[0] == S.greedy(x)
    idx, w, mode = S.candidates(x, True, 1.0, top_k=3, top_p=1.0)
    assert mode == "top_k" and list(idx) == list(np.argsort(-x, kind="stable")[:3])


def test_top_p_cutoff_is_the_first_prefix_reaching_p():  # :439-489
    x = np.log(np.array([0.5, 0.3, 0.15, 0.05]))
    idx, w, _ = S.candidates(x, True, 1.0, top_k=0, top_p=0.79)
    assert list(idx) == [0, 1]  # 0.5 + 0.3 reaches 0.79
    idx, _, _ = S.candidates(x, True, 1.0, top_k=0, top_p=0.81)
    assert list(idx) == [0, 1, 2]


def test_uniform_is_deterministic_and_in_range():
    us = [S.uniform(7, s, r) for s in range(50) for r in range(40)]
    assert all(0.0 <= u < 1.0 for u in us) and len(set(us)) > 1900
    assert S.uniform(7, 3, 5) == S.uniform(7, 3, 5)


def test_sample_tokens_validates_arguments():
    with pytest.raises(T.InvalidArgument) as e:
        T.sample_tokens(None, 8, 1, 8, 16)
    assert "logits is null" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:
        T.sample_tokens(16, 8, 1, 8, None)
    assert "tokens is null" in str(e.value)
    with pytest.raises(T.InvalidArgument):
        T.sample_tokens(16, 8, 1, 0, 16)
    with pytest.raises(T.InvalidArgument):
        T.sample_tokens(16, 8, -1, 8, 16)
    with pytest.raises(T.InvalidArgument) as e:
        T.sample_tokens(16, 4, 2, 8, 16)
    assert "row_stride" in str(e.value)
    T.sample_tokens(16, 8, 0, 8, 16)  # no rows: nothing to do
    with pytest.raises(T.Unsupported) as e:  # one row's slices must fit the cluster's shared memory
        T.sample_tokens(16, 600000, 1, 600000, 16)
    assert "vocab above" in str(e.value)

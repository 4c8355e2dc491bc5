"""The CPU oracle against golden fixtures produced by the reference's own
CUDA code (tests/golden/make_golden.py ran oracle/_ref on a B200 and wrote
these .npz files): decode within |got-ref| <= 2e-3 + 1e-3|ref| of the
reference kernel's fp16 output, append/getCache bytes identical."""
import math
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden as MG  # noqa: E402

DECODE = sorted(GOLDEN.glob("decode_*.npz"))


def test_fixtures_present():
    assert len(DECODE) == len(MG.DECODE_CASES), "golden fixtures missing: run make_golden.py on a GPU"
    assert (GOLDEN / "append_l2_h4_d32.npz").exists()


@pytest.mark.parametrize("path", DECODE, ids=[p.stem for p in DECODE])
def test_oracle_matches_reference_decode_fixture(path):
    f = np.load(path)
    B, Hq, Hkv, S, D, seed = (int(x) for x in f["shape"])
    q, k, v = MG.decode_inputs(B, Hq, Hkv, S, D, seed)
    assert MG.sha(q, k, v) == str(f["input_sha256"]), "input generator drifted"
    ref = O.f16_to_f32(f["out"])
    scale = float(f["scale"])
    assert abs(scale - 1.0 / math.sqrt(D)) < 1e-7
    worst = 0.0
    for b in range(B):
        ours = O.decode_one(q[b], k[b], v[b], scale, eps=1e-6)
        err = np.abs(ours - ref[b])
        assert np.all(err <= 2e-3 + 1e-3 * np.abs(ref[b])), f"{path.stem} b={b} max {err.max():.3e}"
        worst = max(worst, float(err.max()))
    # fp16 output of an fp32 kernel vs fp64: well inside the tolerance
    assert worst < 2e-3


def test_oracle_append_matches_reference_manager_fixture():
    f = np.load(GOLDEN / "append_l2_h4_d32.npz")
    L, H, D, n = (int(x) for x in f["shape"])
    ks = O.normal_f16((L, n, H, D), int(f["seeds"][0]))
    vs = O.normal_f16((L, n, H, D), int(f["seeds"][1]))
    assert MG.sha(ks, vs) == str(f["input_sha256"])
    g = O.geom(L, H, D, 16, 4)
    pool = np.zeros(L * 2 * 4 * 16 * H * D, np.uint16)
    bt = np.array([2], np.int32)
    for lo, hi in ((0, 3), (3, 5)):
        for l in range(L):
            O.append(pool, g, bt, l, lo, ks[l, lo:hi], vs[l, lo:hi])
    for l in range(L):
        k, v = O.gather(pool, g, bt, l, n)
        assert np.array_equal(k, f["k"][l]) and np.array_equal(v, f["v"][l])

"""The CPU oracle reproduces the reference's golden outputs: every open
problem's expected.npz (all five categories, Emmy's own evaluation on the
seeded inputs) within that problem's rtol/atol, with the inputs built by the
runner's seed convention."""
import json

import numpy as np
import pytest

from conftest import PROBLEMS

from emmy_b200.data import materialize
from oracle import expr


@pytest.mark.parametrize("folder", PROBLEMS, ids=lambda p: p.name)
def test_oracle_matches_expected(folder):
    meta = json.loads((folder / "meta.json").read_text())
    k = meta["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    got = expr.evaluate_problem(folder.name, ins)
    exp = np.load(folder / "expected.npz")
    for name, ref in exp.items():
        assert got[name].shape == ref.shape
        assert np.allclose(got[name], ref, rtol=meta["rtol"], atol=meta["atol"]), name
        if meta["rtol"] == 0 and meta["atol"] == 0:
            assert got[name].astype(np.float32).tobytes() == ref.astype(np.float32).tobytes()


def test_bf16_rounding():
    from emmy_b200.data import bf16_bits, bf16_to_f32
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e-39], dtype=np.float32)
    b = bf16_bits(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa (1.0) wins
    assert bf16_to_f32(b)[1] == np.float32(1.0)
    assert bf16_to_f32(b)[2] == np.float32(1.0078125)
    assert bf16_to_f32(b)[3] == np.float32(-2.5)


def test_seed_convention():
    a = {"name": "x", "dtype": "f32", "shape": [8], "seed": 3}
    ref = np.random.default_rng(3).standard_normal([8]).astype(np.float32)
    assert np.array_equal(materialize(a), ref)
    u = {"name": "x", "dtype": "f32", "shape": [8], "seed": 0,
         "dist": {"kind": "uniform", "lo": -1, "hi": 1}}
    assert np.array_equal(materialize(u),
                          np.random.default_rng(0).uniform(-1, 1, [8]).astype(np.float32))

"""Parity on the GPU for the benchmark configurations (IRs written by the
synthesiser in Emmy's schedule forms) against the CPU oracle: small shapes
in full, and the full BASELINE shapes -- the full sum against the float64
sum of all 2^28 inputs, row kernels on sampled rows (rows are independent, so
the oracle of a row is exact) -- plus the size-independent checks the
domain offers (softmax rows sum to 1, L2 rows have unit norm)."""
import numpy as np
import pytest

from emmy_b200 import synth
from emmy_b200.data import materialize
from oracle import expr

pytestmark = pytest.mark.gpu

SMALL = [
    ("vector_add", dict(n=1 << 16)),
    ("vector_add", dict(n=1000, threads=256)),          # ragged: n not a multiple of 8*T
    ("vector_add", dict(n=3, threads=256)),             # fewer elements than threads
    # thin launch (one CTA of 256 per SM): batches of 8 vectors in flight, the
    # last one partial (5 of 8 vectors of some threads exist)
    ("vector_add", dict(n=148 * 256 * 8 * 8 * 2 + 8 * 5 * 256)),
    ("vector_add", dict(n=100_003)),                    # odd n: scalar vectors, batches of 16
    ("full_sum", dict(n=1 << 20, ctas=64)),
    ("full_sum", dict(n=1 << 16, ctas=1, block=128)),   # one CTA (the pinned-coop form)
    ("row_sum", dict(rows=64, cols=2048)),
    ("row_sum", dict(rows=3, cols=8192, block=128)),
    ("row_mean", dict(rows=64, cols=2048)),
    ("rmsnorm", dict(rows=64, cols=1024)),
    ("rmsnorm", dict(rows=16, cols=4096, block=256)),
    ("softmax", dict(rows=64, cols=1024)),
    ("softmax", dict(rows=16, cols=8192, block=128)),   # streamed (not register-resident)
    ("l2norm", dict(rows=64, cols=1024)),
    ("l2norm", dict(rows=8, cols=128, block=32)),       # one warp per row, no tree
]


def _check(p, ins=None, rows=None):
    from emmy_b200 import harness
    g, m = p.build()
    k = m["kernels"][0]
    ins = ins or {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    outs, kern = harness.run(g, m, ins)
    assert kern.kind in ("pointwise", "rows")
    spec = m["oracle"]
    if rows is not None:
        ins = {n: (v[rows] if v.ndim == 2 and v.shape[0] == p.out[1][0] else v)
               for n, v in ins.items()}
    ref = expr.evaluate_family(spec, ins)
    out = spec["output"]
    got = outs[out]
    if rows is not None:
        got = got[rows]
    got = got.reshape(ref[out].shape)
    rtol, atol = expr.tolerance(m, ref[out])
    if rtol == 0 and atol == 0:
        assert got.tobytes() == ref[out].tobytes()
    else:
        assert np.allclose(got, ref[out], rtol=rtol, atol=atol), np.max(np.abs(got - ref[out]))
    return got


@pytest.mark.parametrize("name,kw", SMALL, ids=[f"{n}-{i}" for i, (n, _) in enumerate(SMALL)])
def test_small(name, kw):
    _check(synth.config(name, **kw))


def test_full_sum_baseline():
    _check(synth.full_sum())


@pytest.mark.parametrize("name", ["row_sum", "row_mean", "rmsnorm", "softmax", "l2norm"])
def test_rows_baseline(name):
    p = synth.config(name)
    rows = np.random.default_rng(7).choice(p.out[1][0], 64, replace=False)
    rows.sort()
    got = _check(p, rows=rows)
    if name == "softmax":
        assert np.allclose(got.astype(np.float64).sum(-1), 1.0, atol=1e-4)
    if name == "l2norm":
        assert np.allclose(np.sqrt((got.astype(np.float64) ** 2).sum(-1)), 1.0, atol=1e-4)


def test_vector_add_baseline_bitexact():
    _check(synth.vector_add())

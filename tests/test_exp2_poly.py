"""The FMA-pipe exponential of the attention kernel, checked on the CPU.

``templates.attention.EXP2_POLY`` holds the degree-3 polynomial for 2^f on
[-0.5, 0.5] that some column pairs of the softmax evaluate instead of the MUFU
``ex2`` (``AttentionTemplate._exp2_poly``).  Its header states how it was made
(a linear-programming minimax fit of the relative error on 4001 points) and
its error bound (7.5e-5).  These tests redo the fit, check the bound over a
dense float32 grid with the polynomial evaluated in float32 the way the kernel
does (Horner, one rounding per FMA), and restate the whole emitted sequence
(clamp, Cody-Waite split by the 1.5 * 2^23 shifter, polynomial, exponent
insertion by an integer multiply-add) in numpy against float64 ``exp2``."""
import numpy as np
import pytest

from emmy_b200.templates.attention import EXP2_POLY

BOUND = 7.5e-5
f32 = np.float32


def _horner_f32(f):
    c0, c1, c2, c3 = (f32(c) for c in EXP2_POLY)
    p = (c3 * f + c2).astype(f32)
    p = (p * f + c1).astype(f32)
    return (p * f + c0).astype(f32)


def test_coefficients_are_the_minimax_fit():
    linprog = pytest.importorskip("scipy.optimize").linprog
    n = 4001
    f = np.linspace(-0.5, 0.5, n)
    y = np.exp2(f)
    V = np.vstack([f ** i for i in range(4)]).T / y[:, None]
    # minimise t subject to |V c - 1| <= t at every point
    A = np.vstack([np.hstack([V, -np.ones((n, 1))]), np.hstack([-V, -np.ones((n, 1))])])
    b = np.concatenate([np.ones(n), -np.ones(n)])
    cost = np.zeros(5)
    cost[-1] = 1.0
    r = linprog(cost, A_ub=A, b_ub=b, bounds=[(None, None)] * 4 + [(0, None)], method="highs")
    assert r.success
    # the LP optimum is flat near its minimum: solver versions land on
    # coefficients a few 1e-6 apart with the same maximum error
    assert np.allclose(r.x[:4], np.asarray(EXP2_POLY), rtol=5e-5, atol=0)
    assert r.x[4] < BOUND


def test_polynomial_error_bound_in_float32():
    f = np.linspace(-0.5, 0.5, 400001).astype(f32)
    p = _horner_f32(f).astype(np.float64)
    rel = np.abs(p / np.exp2(f.astype(np.float64)) - 1.0)
    assert rel.max() < BOUND, rel.max()


def _exp2_emitted(x):
    """The PTX sequence of ``_exp2_poly`` restated: max with -126, n by the
    float shifter, f = x - n, Horner, then n * 2^23 added to the bits of p."""
    x = np.maximum(np.asarray(x, f32), f32(-126.0))
    magic = np.array([0x4B400000], np.uint32).view(f32)[0]
    j = (x + magic).astype(f32)
    n = (j - magic).astype(f32)
    f = (x - n).astype(f32)
    p = _horner_f32(f)
    bits = (j.view(np.uint32).astype(np.uint64) * 8388608 + p.view(np.uint32)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(f32)


def test_emitted_sequence_against_float64():
    # the softmax feeds s * log2(e) - m: at most 0, and far below it for
    # scores that vanish
    x = np.concatenate([np.linspace(-125.0, 0.0, 2_000_001),
                        -np.random.default_rng(0).exponential(3.0, 200_000)]).astype(f32)
    x = x[x >= -125.0]
    got = _exp2_emitted(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < BOUND, (rel.max(), x[np.argmax(rel)])
    # below the clamp the result is tiny, never a wrapped exponent
    low = np.array([-126.0, -130.0, -1e4, -np.inf], f32)
    out = _exp2_emitted(low).astype(np.float64)
    assert np.all(np.isfinite(out)) and np.all(out >= 0) and np.all(out < 2.0 ** -124)

"""The reference's 85-IR regression corpus on the GPU: every IR the compiler
accepts runs once on seeded inputs (the reference runner's convention) and its
output must match the expected values committed by make_corpus.py — the
reference's own numpy references (``tools/harness/refs.py``) or, for the five
IRs its compiler rejects, their restated math — with the reference
regression's check ``np.allclose(got, ref, rtol, atol)`` and meta's
tolerances (reference ``tools/harness/regression.py:97-101``).  Each case runs
through the normal template selection and again through the
statement-by-statement lowering alone."""
import json

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

CORPUS = REPO / "tests" / "golden" / "corpus"
INDEX = json.loads((CORPUS / "CORPUS.json").read_text())
NAMES = sorted(n for n, v in INDEX.items() if "refused" not in v)


@pytest.mark.parametrize("mode", ["select", "generic"])
@pytest.mark.parametrize("name", NAMES)
def test_corpus_case(name, mode, monkeypatch):
    from emmy_b200 import harness
    from emmy_b200.data import bf16_to_f32
    if mode == "generic":
        monkeypatch.setenv("EMMY_TEMPLATE", "generic")
    g = json.loads((CORPUS / name / "kernel.ir.json").read_text())
    meta = json.loads((CORPUS / name / "meta.json").read_text())
    outs, kern = harness.run(g, meta, folder=CORPUS / name)
    if mode == "generic":
        assert kern.kind == "generic"
    out = next(a for a in meta["kernels"][0]["args"] if a.get("output"))
    got = outs[out["name"]]
    if out["dtype"] == "bf16":
        got = bf16_to_f32(got)
    got = np.asarray(got).astype(np.float64).reshape(-1)
    exp = np.load(CORPUS / name / "expected.npz")
    ref = exp["val"].astype(np.float64).reshape(-1)
    if "idx" in exp:
        got = got[exp["idx"]]
    assert got.shape == ref.shape
    ok = np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"])
    err = float(np.max(np.abs(got - ref))) if got.size else 0.0
    assert ok, f"{name} ({kern.kind}): max abs err {err:.3e}"

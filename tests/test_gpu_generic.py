"""Parity on the GPU for the statement-by-statement lowering (the path every
IR no template accepts takes):

* all 15 open problems compiled through it (templates disabled) against
  their expected.npz within each problem's rtol/atol;
* the 8 bug fixtures against their frozen ref.bin with the reference's own
  comparison (tools/harness/gpu_check.py: the last output read as f32,
  |got - ref| <= atol + rtol*|ref|; partial_dyn_inv's frozen output carries
  a known 128-element residual, reference tests/expectations.json)."""
import json

import numpy as np
import pytest

from conftest import FIXTURES, PROBLEMS

pytestmark = pytest.mark.gpu


def _expected_ok(outs, folder, meta):
    exp = np.load(folder / "expected.npz")
    for name, ref in exp.items():
        got = outs[name].reshape(ref.shape)
        if meta["rtol"] == 0 and meta["atol"] == 0:
            assert got.tobytes() == ref.astype(np.float32).tobytes(), name
        else:
            err = np.max(np.abs(got.astype(np.float64) - ref))
            assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]), (name, err)


@pytest.mark.parametrize("folder", PROBLEMS, ids=lambda p: p.name)
def test_problem_generic(folder, monkeypatch):
    from emmy_b200 import harness
    monkeypatch.setenv("EMMY_TEMPLATE", "generic")
    g = json.loads((folder / "kernel.ir.json").read_text())
    meta = json.loads((folder / "meta.json").read_text())
    outs, kern = harness.run(g, meta)
    assert kern.kind == "generic"
    _expected_ok(outs, folder, meta)


@pytest.mark.parametrize("folder", FIXTURES, ids=lambda p: p.name)
def test_fixture(folder):
    from emmy_b200 import harness
    g = json.loads((folder / "kernel.ir.json").read_text())
    meta = json.loads((folder / "meta.json").read_text())
    outs, kern = harness.run(g, meta, folder=folder)
    k = meta["kernels"][0]
    last = [a["name"] for a in k["args"] if a.get("output")][-1]
    got_b = outs[last].tobytes()
    ref_b = (folder / "ref.bin").read_bytes()
    n = min(len(got_b), len(ref_b)) // 4
    got = np.frombuffer(got_b[:4 * n], dtype=np.float32).astype(np.float64)
    ref = np.frombuffer(ref_b[:4 * n], dtype=np.float32).astype(np.float64)
    if folder.name == "smem_align":
        # add[5] is computed from s[6], a shared-memory word no thread of this
        # IR writes (thread a0=2 reads s[2*a0+2]); its frozen value is whatever
        # that run's shared memory held, so only add[0..4] are defined
        got, ref = got[:5], ref[:5]
    with np.errstate(invalid="ignore"):
        bad = int(np.sum(np.abs(got - ref) > meta["atol"] + meta["rtol"] * np.abs(ref)))
    allowed = 128 if folder.name == "partial_dyn_inv" else 0
    assert bad <= allowed, f"{bad} elements outside tolerance ({kern.kind})"

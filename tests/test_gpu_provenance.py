"""On the GPU, the two lowering fixes the static checkers led to, through
the statement-by-statement lowering:

* ``Let first = acc`` before a loop that accumulates into ``acc`` keeps the
  value ``first`` was bound to (an SSA binding): ``y = first + acc`` equals
  the f32 sum ``x + x + x + x`` bit for bit (an aliasing ``Let`` gives
  ``2 * acc``);
* the warp-indexed ``TreeHalve`` (the reference's reduction form) stores from
  one lane after a warp barrier: the golden problems that use it match their
  expected outputs (also run by the corpus and problem tests; repeated here
  for the form the race checker flagged)."""
import json

import numpy as np
import pytest

from conftest import PROBLEMS

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("inside", [False, True], ids=["after-loop", "in-loop"])
def test_let_is_ssa(inside, monkeypatch):
    from emmy_b200 import harness
    from test_provcheck import _let_alias
    monkeypatch.setenv("EMMY_TEMPLATE", "generic")
    g, m = _let_alias(read_inside_loop=inside).build()
    x = np.random.default_rng(5).standard_normal(1024).astype(np.float32)
    outs, kern = harness.run(g, m, {"x": x})
    assert kern.kind == "generic"
    acc = np.zeros_like(x)
    for _ in range(4):
        acc = (acc + x).astype(np.float32)
    assert np.array_equal(outs["y"], acc), float(np.max(np.abs(outs["y"] - acc)))


@pytest.mark.parametrize("pid", ["r01_array_sum", "r04_row_sum", "f02_row_softmax"])
def test_warp_tree_problems(pid, monkeypatch):
    from emmy_b200 import harness
    monkeypatch.setenv("EMMY_TEMPLATE", "generic")
    folder = next(p for p in PROBLEMS if p.name == pid)
    g = json.loads((folder / "kernel.ir.json").read_text())
    m = json.loads((folder / "meta.json").read_text())
    assert "tid_var='warp'" in json.dumps(g)
    outs, kern = harness.run(g, m, folder=folder)
    assert kern.kind == "generic"
    exp = np.load(folder / "expected.npz")
    for name in exp.files:
        ref = exp[name]
        got = outs[name].reshape(ref.shape)
        assert np.allclose(got, ref, rtol=m.get("rtol", 1e-4), atol=m.get("atol", 1e-5)), name

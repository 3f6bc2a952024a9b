"""The IR nodes the vocabulary defines and no reference IR uses (the reference
compiler exits 1 on them; reference TASK.md rows marked *): ``Pre``/``Carry``,
``Select`` and ``ZeroPrologue`` lowered by the statement-by-statement path,
on IRs written from the table's own descriptions (``synth.carried_prefix``,
``select_branches``, ``zero_prologue``), against the oracle restated from the
same descriptions."""
import numpy as np
import pytest

from emmy_b200 import synth
from emmy_b200.data import materialize
from oracle import expr

pytestmark = pytest.mark.gpu


def _run(p, prefill=None):
    import torch
    from emmy_b200 import harness, native
    g, m = p.build()
    kern = harness.CompiledKernel(g, m)
    assert kern.kind == "generic"
    k = m["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    bufs = harness.Buffers(kern, ins)
    if prefill is not None:
        for a in k["args"]:
            if a.get("output"):
                bufs.t[a["name"]].fill_(prefill)
    stream = torch.cuda.current_stream().cuda_stream
    kern.launch(bufs.ptrs(), stream)
    torch.cuda.synchronize()
    outs = bufs.outputs()
    spec = m["oracle"]
    ref = expr.evaluate_family(spec, ins)[spec["output"]]
    got = outs[spec["output"]].reshape(ref.shape)
    rtol, atol = expr.tolerance(m, ref)
    if rtol == 0 and not atol:
        assert got.tobytes() == ref.tobytes()
    else:
        assert np.allclose(got, ref, rtol=rtol, atol=atol), float(np.max(np.abs(got - ref)))


@pytest.mark.parametrize("kw", [dict(cols=96, every=1), dict(cols=96, every=2),
                                dict(cols=200, every=3), dict(rows=100, cols=40, every=5)],
                         ids=["unrolled", "skips", "loop", "ragged"])
def test_carry_and_pre(kw):
    """Steps read the previous state (the seed first), skipped steps keep the
    cell; 96 and 40 columns are unrolled, 200 stay a loop; 100 rows over
    64-thread CTAs leave idle threads."""
    _run(synth.carried_prefix(**kw))


def test_select():
    _run(synth.select_branches())


def test_zero_prologue():
    """The output starts as 7.0 everywhere: the kernel zeroes its first
    ``words`` words itself, then adds its inputs atomically."""
    _run(synth.zero_prologue(), prefill=7.0)

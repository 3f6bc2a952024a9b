"""Parity on the GPU against the reference's golden vectors: each open
problem compiled by compile.py, launched through the C ABI under its own
meta.json, and compared with the problem's expected.npz within the problem's
rtol/atol (pointwise problems: bit for bit)."""
import json

import numpy as np
import pytest

from conftest import PROBLEMS

pytestmark = pytest.mark.gpu

SUPPORTED = {p.name for p in PROBLEMS}   # templates where they apply, else the generic path


@pytest.mark.parametrize("folder", [p for p in PROBLEMS if p.name in SUPPORTED],
                         ids=lambda p: p.name)
def test_problem_matches_expected(folder):
    from emmy_b200 import harness
    g = json.loads((folder / "kernel.ir.json").read_text())
    meta = json.loads((folder / "meta.json").read_text())
    outs, kern = harness.run(g, meta)
    exp = np.load(folder / "expected.npz")
    for name, ref in exp.items():
        got = outs[name].reshape(ref.shape)
        if meta["rtol"] == 0 and meta["atol"] == 0:
            assert got.tobytes() == ref.astype(np.float32).tobytes(), name
        else:
            err = np.max(np.abs(got.astype(np.float64) - ref))
            assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]), (name, err)


@pytest.mark.parametrize("folder", [p for p in PROBLEMS if p.name in SUPPORTED],
                         ids=lambda p: p.name)
def test_problem_repeat_launch(folder):
    """Two launches on the same buffers give the same result (outputs in
    zero_outputs are re-zeroed; nothing else carries state)."""
    import torch
    from emmy_b200 import harness, native
    g = json.loads((folder / "kernel.ir.json").read_text())
    meta = json.loads((folder / "meta.json").read_text())
    kern = harness.CompiledKernel(g, meta)
    bufs = harness.Buffers(kern)
    s = torch.cuda.current_stream().cuda_stream
    res = []
    for _ in range(2):
        for z, nb in bufs.zero_list():
            native.check(native.lib().emmy_memset_async(z, 0, nb, s))
        kern.launch(bufs.ptrs(), s)
        torch.cuda.synchronize()
        res.append({k: v.copy() for k, v in bufs.outputs().items()})
    for k in res[0]:
        if kern.ctx.zero_outputs or k not in [a["name"] for a in meta["kernels"][0]["args"]
                                              if a.get("output")]:
            continue
        assert np.array_equal(res[0][k], res[1][k])

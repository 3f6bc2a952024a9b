"""The TMA / mbarrier statements of the IR on the GPU: box copies through
shared memory (mbarrier slots declared as Smem or implied) give exactly
``2 x + 1``; an mbarrier wait that nothing completes gives up after its 2 s
bound with status 8 and the kernel still finishes -- the failure path is
exercised without a fault or a hang."""
import numpy as np
import pytest

from emmy_b200 import synth

pytestmark = pytest.mark.gpu


def _run(p):
    import torch
    from emmy_b200 import harness, native
    from emmy_b200.data import materialize
    g, m = p.build()
    k = m["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    outs, kern = harness.run(g, m, ins)
    addr, _ = kern.module().global_addr("__emmy_status")
    st = torch.zeros(1, dtype=torch.int32)
    native.check(native.lib().emmy_memcpy_dtoh_async(st.data_ptr(), addr, 4, None))
    torch.cuda.synchronize()
    return ins, outs, int(st[0])


@pytest.mark.parametrize("kw", [dict(), dict(boxes=1, declare_mbar=False),
                                dict(box_rows=16, box_cols=32, boxes=4, rows=1024)])
def test_tma_scale(kw):
    ins, outs, status = _run(synth.tma_scale(**kw))
    assert status == 0
    x = ins["x"].astype(np.float32)
    ref = (x * np.float32(2.0) + np.float32(1.0)).astype(np.float32)
    assert outs["y"].reshape(ref.shape).tobytes() == ref.tobytes()


def test_mbarrier_wait_times_out_cleanly():
    ins, outs, status = _run(synth.mbarrier_timeout())
    assert status == 8
    assert outs["y"].tobytes() == ins["x"].astype(np.float32).tobytes()

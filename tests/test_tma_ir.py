"""The TMA / mbarrier / SetMaxNReg statements (defined by the reference's IR,
TASK.md "Transport into shared memory", never lowered by it), on the CPU:
they compile through the generic lowering to PTX ptxas accepts; every bulk
tensor copy is preceded by the run-time alignment guard on its shared-memory
destination; compile-time violations of the TMA rules are refused; SetMaxNReg
emits no setmaxnreg (it is a hint whose .inc could wait forever)."""
import re

import pytest

from emmy_b200 import ir as I
from emmy_b200 import synth


def _ptx(p):
    from emmy_b200 import native
    from emmy_b200.compiler import compile_graph
    g, m = p.build()
    c = compile_graph(g, m)
    ptx = c.render()
    assert c.kind == "generic"
    native.Image(ptx)
    return ptx


@pytest.mark.parametrize("kw", [dict(), dict(boxes=1), dict(declare_mbar=False),
                                dict(box_rows=16, box_cols=32, boxes=4)])
def test_tma_scale_compiles_guarded(kw):
    ptx = _ptx(synth.tma_scale(**kw))
    lines = ptx.splitlines()
    copies = [i for i, ln in enumerate(lines) if "cp.async.bulk.tensor" in ln]
    assert len(copies) == kw.get("boxes", 2)
    for i in copies:
        window = "\n".join(lines[max(0, i - 8):i])
        assert re.search(r"and\.b32 %r\d+, %r\d+, 127;", window), window
    assert "setmaxnreg" not in ptx.replace("SetMaxNReg", "")
    assert "// @emmy tmap tmap_xd buf=x dtype=7" in ptx
    assert ".param .align 64 .b8 param_tmap_xd[128]" in ptx
    # every wait is bounded
    assert ptx.count("mbarrier.try_wait.parity") == 2 * ptx.count("%globaltimer;") // 2


def test_tma_misaligned_literal_x_refused():
    p = synth.tma_scale(boxes=1)
    body = list(p.body.body)
    for i, s in enumerate(body):
        if type(s).__name__ == "Cond" and any(type(t).__name__ == "TmaLoad" for t in s.body):
            st = tuple(I.TmaLoad(t.smem, t.smem_index, t.desc, (t.coords[0], synth.Lit(3)),
                                 t.mbar, t.mbar_slot) if type(t).__name__ == "TmaLoad" else t
                       for t in s.body)
            body[i] = I.Cond(s.cond, st, s.else_body)
    p.body = synth.tile(list(p.body.axes), body)
    with pytest.raises(NotImplementedError, match="16-byte aligned"):
        _ptx(p)


def test_tma_descriptor_beyond_buffer_refused():
    p = synth.tma_scale(boxes=1)
    body = [I.TmaDescriptor(s.name, s.src_buf, (4096, 64), s.box_extents, s.swizzle, s.dtype)
            if type(s).__name__ == "TmaDescriptor" else s for s in p.body.body]
    p.body = synth.tile(list(p.body.axes), body)
    with pytest.raises(NotImplementedError, match="exceeds buffer"):
        _ptx(p)


def test_mbarrier_timeout_compiles():
    ptx = _ptx(synth.mbarrier_timeout())
    assert "mbarrier.init.shared::cta.b64" in ptx and "st.global.u32 [%rd" in ptx

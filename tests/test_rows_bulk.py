"""The one-CTA streaming sums' bulk-copy ring (templates/rows.py): which
launches take it, and the shape of what it emits -- one 1-D bulk copy per
batch of the row (no tensor map, no multicast), at most three stages of
static shared memory within the 48 KiB a launcher allows, every wait on a
stage bounded -- checked on the compiled PTX of the reference's own r02/r03
IRs and of synthesised sums."""
import json
import re

import pytest

from conftest import GOLDEN
from emmy_b200 import ptxcheck, synth
from emmy_b200.compiler import compile_graph
from emmy_b200.templates import rows

COPY = "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"


def _ptx(pid):
    f = GOLDEN / "problems" / pid
    c = compile_graph(json.loads((f / "kernel.ir.json").read_text()),
                      json.loads((f / "meta.json").read_text()))
    return c.kind, c.render()


@pytest.mark.parametrize("pid,J", [("r02_big_sum", 64), ("r03_mean", 32)])
def test_problem_sums_stream_through_the_bulk_ring(pid, J):
    kind, ptx = _ptx(pid)
    assert kind == "rows"
    per = 128 * 8 * 4                                  # one vector of every thread
    batch = rows.BULK_STAGE // per
    assert ptx.count(COPY) == -(-J // batch)           # one copy per batch, unrolled
    assert "multicast" not in ptx and "tensormap" not in ptx
    stage = int(re.search(r"__emmy_bulk\[(\d+)\]", ptx).group(1))
    assert stage == rows.BULK_STAGES * batch * per <= 48 * 1024
    assert ptx.count("mbarrier.try_wait") == 2 * -(-J // batch)   # first try + bounded loop
    assert ptxcheck.check(ptx) == []


def test_wide_ctas_keep_the_register_stream():
    # one vector of each of 1024 threads is 32 KiB, more than a stage
    g, m = synth.config("full_sum", n=1 << 20, ctas=1, block=1024).build()
    assert COPY not in compile_graph(g, m).render()


def test_many_cta_launches_do_not_use_it():
    g, m = synth.config("full_sum", n=1 << 20, ctas=256).build()
    assert COPY not in compile_graph(g, m).render()

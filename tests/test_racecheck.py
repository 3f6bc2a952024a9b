"""The shared-memory race checker (``emmy_b200.racecheck``), the static
substitute for compute-sanitizer's racecheck (reference
``tools/checkers/racecheck.py``): every kernel this build generates is free
of races, the templates' shared-memory accesses are all resolved (none left
to the ``unresolved`` count), and races planted into real generated PTX, or
written into small kernels by hand, are found with a concrete thread pair."""
import json
import os
import re

import pytest

from conftest import PROBLEMS

from emmy_b200 import racecheck, synth
from emmy_b200.compiler import compile_graph

SMALL = {"vector_add": dict(n=1 << 16), "full_sum": dict(n=1 << 20, ctas=64),
         "row_sum": dict(rows=64, cols=2048), "row_mean": dict(rows=64, cols=2048),
         "rmsnorm": dict(rows=64, cols=1024), "softmax": dict(rows=64, cols=1024),
         "l2norm": dict(rows=64, cols=1024), "matmul_bf16": dict(M=256, N=256, K=128),
         "matmul_f32": dict(M=256, N=256, K=128), "attention": dict(B=1, H=2, S=512),
         "attention_d64": dict(B=1, H=2, S=512)}


def _threads(m):
    b = m["kernels"][0]["block"]
    return b[0] * b[1] * b[2]


def _ptx(name, generic=False, monkeypatch=None, **kw):
    if generic:
        monkeypatch.setenv("EMMY_TEMPLATE", "generic")
    g, m = synth.config(name, **kw).build()
    return compile_graph(g, m).render(), m


@pytest.mark.parametrize("name", sorted(SMALL))
def test_templates_race_free_and_resolved(name):
    for kw in ({}, SMALL[name]):
        ptx, m = _ptx(name, **kw)
        races, st = racecheck.check(ptx, threads=_threads(m))
        assert races == [], races[:2]
        assert st["unresolved"] == 0, st


def test_goldens_race_free_both_paths(monkeypatch):
    for forced in (None, "generic"):
        if forced:
            monkeypatch.setenv("EMMY_TEMPLATE", forced)
        for folder in PROBLEMS:
            g = json.loads((folder / "kernel.ir.json").read_text())
            m = json.loads((folder / "meta.json").read_text())
            races, _ = racecheck.check(compile_graph(g, m).render(), threads=_threads(m))
            assert races == [], (folder.name, forced, races[:2])


def _drop_barrier_after(ptx, marker):
    """Remove the first CTA barrier following the first line containing marker."""
    lines = ptx.splitlines()
    i = next(n for n, ln in enumerate(lines) if marker in ln)
    j = next(n for n in range(i, len(lines)) if re.match(r"\s*(bar|barrier)\.sync", lines[n]))
    return "\n".join(lines[:j] + lines[j + 1:])


def test_plant_missing_barrier_in_rows_template():
    """rmsnorm: lane 0 of each warp stores its warp's partial, a CTA barrier,
    then every thread reads the partials; without the barrier a reader races
    with a writer of another warp."""
    ptx, m = _ptx("rmsnorm", rows=64, cols=1024)
    assert racecheck.check(ptx, threads=_threads(m))[0] == []
    bad = _drop_barrier_after(ptx, "st.shared")
    races, _ = racecheck.check(bad, threads=_threads(m))
    assert races and all(r[2] >> 5 != r[3] >> 5 for r in races), races[:2]


def test_plant_warp_redundant_tree_store(monkeypatch):
    """The generic TreeHalve over warp indices: without its lane-0 store
    predicate all 32 lanes write the same entry (write/write); without its
    warp barrier a lane's store can overtake another lane's load."""
    monkeypatch.setenv("EMMY_TEMPLATE", "generic")
    folder = next(p for p in PROBLEMS if p.name == "r01_array_sum")
    g = json.loads((folder / "kernel.ir.json").read_text())
    m = json.loads((folder / "meta.json").read_text())
    ptx = compile_graph(g, m).render()
    n = _threads(m)
    assert racecheck.check(ptx, threads=n)[0] == []
    no_pred = re.sub(r"@%p\d+ (st\.shared)", r"\1", ptx)
    races, _ = racecheck.check(no_pred, threads=n)
    assert any(r[5].startswith("W/W") for r in races), races[:2]
    no_sync = re.sub(r"\tbar\.warp\.sync %r\d+;\n", "", ptx)
    races, _ = racecheck.check(no_sync, threads=n)
    assert any(r[5].startswith(("R/W", "W/R")) and r[2] >> 5 == r[3] >> 5 for r in races), \
        races[:2]


_HAND = """.version 8.8
.target sm_100a
.address_size 64
.shared .align 4 .b8 buf[1024];
.visible .entry k()
.maxntid 128, 1, 1
{{
\t.reg .b32 %r<9>;
\t.reg .pred %p<3>;
\t.reg .f32 %f<3>;
\tmov.u32 %r1, %tid.x;
\tmov.u32 %r2, buf;
\tmov.f32 %f1, 0f3F800000;
{body}
\tret;
}}
"""


@pytest.mark.parametrize("body,racy", [
    # every thread stores its own word
    ("\tmad.lo.u32 %r3, %r1, 4, %r2;\n\tst.shared.f32 [%r3], %f1;", False),
    # every thread stores the same word
    ("\tst.shared.f32 [%r2], %f1;", True),
    # only thread 0 stores it
    ("\tsetp.eq.u32 %p1, %r1, 0;\n\t@%p1 st.shared.f32 [%r2], %f1;", False),
    # thread t writes word t, reads word t+1 in the same region
    ("\tmad.lo.u32 %r3, %r1, 4, %r2;\n\tst.shared.f32 [%r3], %f1;\n"
     "\tld.shared.f32 %f2, [%r3+4];", True),
    # ... with a CTA barrier in between
    ("\tmad.lo.u32 %r3, %r1, 4, %r2;\n\tst.shared.f32 [%r3], %f1;\n\tbar.sync 0;\n"
     "\tld.shared.f32 %f2, [%r3+4];", False),
    # lane 0 of each warp writes word[warp]; a warp-only barrier does not
    # order another warp's read of it
    ("\tshr.u32 %r4, %r1, 5;\n\tand.b32 %r5, %r1, 31;\n\tsetp.eq.u32 %p1, %r5, 0;\n"
     "\tmad.lo.u32 %r6, %r4, 4, %r2;\n\t@%p1 st.shared.f32 [%r6], %f1;\n"
     "\tbar.warp.sync 0xffffffff;\n\tld.shared.f32 %f2, [%r2+4];", True),
    # ... and reading its own warp's word after the warp barrier is fine
    ("\tshr.u32 %r4, %r1, 5;\n\tand.b32 %r5, %r1, 31;\n\tsetp.eq.u32 %p1, %r5, 0;\n"
     "\tmad.lo.u32 %r6, %r4, 4, %r2;\n\t@%p1 st.shared.f32 [%r6], %f1;\n"
     "\tbar.warp.sync 0xffffffff;\n\tld.shared.f32 %f2, [%r6];", False),
    # atomics on one word do not race with each other
    ("\tatom.shared.add.f32 %f2, [%r2], %f1;", False),
])
def test_hand_written(body, racy):
    races, st = racecheck.check(_HAND.format(body=body))
    assert bool(races) == racy, races
    assert st["unresolved"] == 0


def test_cli(tmp_path):
    from emmy_b200.racecheck import main
    f = tmp_path / "k.ptx"
    f.write_text(_HAND.format(body="\tst.shared.f32 [%r2], %f1;"))
    assert main([str(f)]) == 1
    f.write_text(_HAND.format(body="\tmad.lo.u32 %r3, %r1, 4, %r2;\n\tst.shared.f32 [%r3], %f1;"))
    assert main([str(f)]) == 0

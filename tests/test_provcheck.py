"""The IR-name provenance checker (``emmy_b200.provcheck``; reference
``tools/checkers/provcheck.py``) over the statement-by-statement lowering:
every golden IR (problems, fixtures, the 85-IR corpus) lowers without a name
observing another name's in-place update, and the hazard the checker exists
for -- ``Let a = acc`` followed by ``Accum acc`` and a read of ``a`` -- is
reported when the lowering aliases the two names (planted here by
restoring an aliasing ``Let``), later in the program and across loop
iterations, and is absent with the lowering's copying ``Let``."""
import json

import pytest

from conftest import FIXTURES, PROBLEMS, REPO

from emmy_b200 import generic, provcheck
from emmy_b200 import ir as I
from emmy_b200 import synth as S

CORPUS = sorted(p for p in (REPO / "tests/golden/corpus").iterdir() if p.is_dir())


def _let_alias(read_inside_loop=False, n=1024, block=128):
    """``first = acc`` (Let) before a loop that accumulates x into acc; the
    IR's SSA meaning: first == 0 and acc == 4x.  With ``read_inside_loop``,
    ``first`` is read in the loop body (each iteration must see 0)."""
    p = S.Problem(f"let_alias_{n}", "x", "k_let_alias", "y")
    p.add_input("x", (n,))
    p.out = ("y", (n,), "f32")
    if read_inside_loop:                  # acc += first + x
        inner = [S.load("in0", "x", S.V("a0")), S.assign("t", "add", "first", "in0"),
                 S.accum("acc", "t", axes=("j",))]
    else:                                 # acc += x
        inner = [S.load("in0", "x", S.V("a0")), S.accum("acc", "in0", axes=("j",))]
    body = [I.Init("acc", 0.0, S.F32), I.Let("first", S.V("acc"), S.F32),
            I.Loop(S.axis("j", 4), tuple(inner), False, False),
            S.assign("out", "add", "first", "acc"),
            S.write("y", (S.V("a0"),), ("out",))]
    p.body = S.tile([S.axis("a0", n)], body)
    p.grid, p.block = (n // block, 1, 1), (block, 1, 1)
    return p


def _aliasing_let(self, s):
    """The lowering before the fix: Let of a name shares its register."""
    if type(s.value).__name__ == "Var" and s.value.name in self.vals:
        self.vals[s.name] = self.vals[s.value.name]
        return
    return _ORIG_LET(self, s)


_ORIG_LET = generic.GenericLowering.s_Let


@pytest.mark.parametrize("folders", [PROBLEMS, FIXTURES, CORPUS], ids=["problems", "fixtures",
                                                                    "corpus"])
def test_goldens_clean(folders):
    checked = 0
    for folder in folders:
        g = json.loads((folder / "kernel.ir.json").read_text())
        m = json.loads((folder / "meta.json").read_text())
        try:
            v, _, _ = provcheck.check_graph(g, m)
        except NotImplementedError:
            continue                      # IRs the lowering refuses (exit 1)
        assert v == [], (folder.name, v)
        checked += 1
    assert checked >= len(folders) - 1


@pytest.mark.parametrize("inside", [False, True], ids=["after-loop", "in-loop"])
def test_let_alias_planted_and_fixed(inside, monkeypatch):
    g, m = _let_alias(read_inside_loop=inside).build()
    v, _, _ = provcheck.check_graph(g, m)
    assert v == []
    monkeypatch.setattr(generic.GenericLowering, "s_Let", _aliasing_let)
    v, _, _ = provcheck.check_graph(g, m)
    assert v and v[0][:2] == ("first", "acc"), v


def test_benign_alias_not_reported(monkeypatch):
    """An alias whose source is never updated afterwards is benign."""
    monkeypatch.setattr(generic.GenericLowering, "s_Let", _aliasing_let)
    p = S.Problem("let_plain", "x", "k_let_plain", "y")
    p.add_input("x", (1024,))
    p.out = ("y", (1024,), "f32")
    p.body = S.tile([S.axis("a0", 1024)], [
        S.load("in0", "x", S.V("a0")), I.Let("c", S.V("in0"), S.F32),
        S.assign("o", "add", "c", "in0"), S.write("y", (S.V("a0"),), ("o",))])
    p.grid, p.block = (8, 1, 1), (128, 1, 1)
    g, m = p.build()
    v, benign, _ = provcheck.check_graph(g, m)
    assert v == [] and [b[:2] for b in benign] == [("c", "in0")]


def test_cli(tmp_path):
    g, m = _let_alias().build()
    d = tmp_path / "let_alias"
    d.mkdir()
    (d / "kernel.ir.json").write_text(json.dumps(g))
    (d / "meta.json").write_text(json.dumps(m))
    assert provcheck.main([str(tmp_path)]) == 0

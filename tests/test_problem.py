"""Problem folders and the submit flow, on the CPU: the multi-kernel
``Pipeline`` writes the reference's layout (``<entry>.ir.json`` per kernel,
``meta.json`` with seeds by graph-input position, ``data`` constants,
``intermediate`` arguments for buffers an earlier kernel writes, ``final`` on
kernels that write a graph output; reference ``tools/generate.py:108-146``),
every kernel of it compiles, and ``submit.py`` refuses bad command lines with
the reference's messages and exit codes."""
import json
import subprocess
import sys

import pytest

from conftest import REPO


@pytest.mark.parametrize("build", ["rmsnorm_two_kernel", "softmax_three_kernel"])
def test_pipeline_layout(build, tmp_path):
    from emmy_b200 import native, synth
    from emmy_b200.compiler import compile_graph
    pl = getattr(synth, build)()
    folder = pl.write(tmp_path / pl.pid)
    meta = json.loads((folder / "meta.json").read_text())
    assert len(meta["kernels"]) >= 2
    produced = set()
    for i, k in enumerate(meta["kernels"]):
        assert (folder / f"{k['entry']}.ir.json").exists()
        assert k["arg_order"] == [a["name"] for a in k["args"]]
        for a in k["args"]:
            if a.get("intermediate"):
                assert a["name"] in produced
            elif "seed" in a:
                assert meta["graph_inputs"][a["seed"]] == a["name"]
            elif a.get("output"):
                produced.add(a["name"])
        assert k["final"] == (i == len(meta["kernels"]) - 1)
        g = json.loads((folder / f"{k['entry']}.ir.json").read_text())
        assert k["entry"] in native.Image(compile_graph(g, meta).render()).registers()


def test_pipeline_rejects_unknown_buffer():
    from emmy_b200 import synth
    pl = synth.rmsnorm_two_kernel()
    pl.stages = pl.stages[1:]          # the apply kernel alone: nobody writes ms
    with pytest.raises(ValueError, match="neither a graph input"):
        pl.build()


def _submit(*args):
    return subprocess.run([sys.executable, str(REPO / "submit.py"), *args],
                          capture_output=True, text=True, cwd=REPO)


def test_submit_usage_errors(tmp_path):
    from emmy_b200 import synth
    r = _submit()
    assert r.returncode == 2                          # argparse: missing argument
    # the reference's sys.exit(msg): message on stderr, exit 1
    r = _submit("no_such_problem", "--compiler", "compile.py")
    assert r.returncode == 1 and "unknown problem" in r.stderr
    r = _submit("p01_vector_add")
    assert r.returncode == 1 and "give a PTX file or --compiler" in r.stderr
    folder = synth.softmax_three_kernel(rows=4, cols=256).write(tmp_path / "sm3")
    r = _submit(str(folder), "x.ptx")
    assert r.returncode == 1 and "has 3 kernels - use --compiler" in r.stderr


def test_not_ptx():
    from emmy_b200.problem import not_ptx
    assert not_ptx("") == "it is empty"
    assert "instead of a directive" in not_ptx("hello\n.version 8.8")
    assert not_ptx("// comment\n.version 8.8\n.target sm_100a\n") is None

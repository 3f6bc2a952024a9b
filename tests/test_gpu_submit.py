"""The submit flow on the GPU (reference ``submit.py``): every open problem
passes through ``submit.py --compiler compile.py``; multi-kernel problems
chain their intermediates in device memory and match the oracle at the end
and in between; a PTX file works for a single-kernel problem; a problem whose
kernel needs a buffer no earlier kernel wrote is refused."""
import json
import subprocess
import sys

import numpy as np
import pytest

from conftest import PROBLEMS, REPO
from oracle import expr

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("folder", PROBLEMS, ids=lambda p: p.name)
def test_open_problem_through_compiler(folder):
    from emmy_b200 import problem
    lines = []
    rep = problem.run_problem(folder, problem.compiler_ptx(str(REPO / "compile.py")),
                              out=lines.append)
    assert rep["ok"], lines
    assert any("PASS" in ln for ln in lines), lines


def _pipeline_folder(pl, tmp_path):
    from emmy_b200.data import materialize
    irs, meta = pl.build()
    args = {a["name"]: a for k in meta["kernels"] for a in k["args"] if "seed" in a}
    ins = {n: materialize(a) for n, a in args.items()}
    ref = expr.evaluate_family(meta["oracle"], ins)
    return pl.write(tmp_path / pl.pid, {meta["oracle"]["output"]: ref[meta["oracle"]["output"]]}), ins


def test_rmsnorm_two_kernels(tmp_path):
    from emmy_b200 import problem, synth
    folder, ins = _pipeline_folder(synth.rmsnorm_two_kernel(rows=192, cols=1024), tmp_path)
    lines = []
    rep = problem.run_problem(folder, out=lines.append, time_launches=True)
    assert rep["ok"], lines
    assert [k["entry"] for k in rep["kernels"]] == ["k_rms_meansq", "k_rms_apply"]
    x = ins["x"].astype(np.float64)
    ms = (x * x).mean(-1)
    assert np.allclose(rep["outputs"]["ms"], ms, rtol=1e-5, atol=1e-6)


def test_softmax_three_kernels_cli(tmp_path):
    from emmy_b200 import synth
    folder, ins = _pipeline_folder(synth.softmax_three_kernel(rows=64, cols=2048), tmp_path)
    r = subprocess.run([sys.executable, str(REPO / "submit.py"), str(folder), "--compiler",
                        str(REPO / "compile.py")], capture_output=True, text=True, cwd=REPO)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "[k_sm_norm] PASS  softmax" in r.stdout


def test_ptx_file_single_kernel(tmp_path):
    folder = next(p for p in PROBLEMS if p.name == "p01_vector_add")
    ptx = subprocess.run([sys.executable, str(REPO / "compile.py"), str(folder / "kernel.ir.json")],
                         capture_output=True, text=True, check=True).stdout
    (tmp_path / "out.ptx").write_text(ptx)
    r = subprocess.run([sys.executable, str(REPO / "submit.py"), "p01_vector_add",
                        str(tmp_path / "out.ptx")], capture_output=True, text=True, cwd=REPO)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout


def test_missing_intermediate_refused(tmp_path):
    from emmy_b200 import problem, synth
    folder = synth.rmsnorm_two_kernel(rows=8, cols=256).write(tmp_path / "rms")
    meta = json.loads((folder / "meta.json").read_text())
    meta["kernels"] = meta["kernels"][::-1]        # the apply kernel first
    (folder / "meta.json").write_text(json.dumps(meta))
    lines = []
    rep = problem.run_problem(folder, out=lines.append)
    assert not rep["ok"]
    assert "needs ms from an earlier kernel" in lines[-1]

"""The static PTX checker (``emmy_b200.ptxcheck``), the sanitizer substitute
for this build's kernels: every kernel the compiler generates (templates,
generic lowering, the reference corpus, TMA IRs) is clean, and each rule
fires on a defect planted in real generated PTX (text edits on the CPU; no
planted kernel is ever launched)."""
import json
import re

import pytest

from emmy_b200 import ptxcheck

from conftest import PROBLEMS, REPO

CONFIGS = ["vector_add", "full_sum", "row_sum", "row_mean", "rmsnorm", "softmax", "l2norm",
           "matmul_bf16", "matmul_f32", "attention", "attention_d64"]
CORPUS = REPO / "tests" / "golden" / "corpus"


def _ptx_config(name, **kw):
    from emmy_b200 import synth
    from emmy_b200.compiler import compile_graph
    g, m = synth.config(name, **kw).build()
    return compile_graph(g, m).render()


def _ptx_folder(d, ir="kernel.ir.json"):
    from emmy_b200.compiler import compile_graph
    return compile_graph(json.loads((d / ir).read_text()),
                         json.loads((d / "meta.json").read_text())).render()


def _rules(ptx):
    from emmy_b200 import ptxcheck
    return [f[0] for f in ptxcheck.check(ptx)]


@pytest.mark.parametrize("name", CONFIGS)
def test_configs_clean(name):
    assert _rules(_ptx_config(name)) == []


@pytest.mark.parametrize("folder", PROBLEMS, ids=lambda p: p.name)
def test_problems_clean(folder):
    assert _rules(_ptx_folder(folder)) == []


def test_corpus_clean():
    idx = json.loads((CORPUS / "CORPUS.json").read_text())
    bad = {n: _rules(_ptx_folder(CORPUS / n)) for n, v in idx.items() if "refused" not in v}
    assert not {n: r for n, r in bad.items() if r}


def test_tma_irs_clean():
    from emmy_b200 import synth
    from emmy_b200.compiler import compile_graph
    for p in (synth.tma_scale(), synth.tma_scale(declare_mbar=False), synth.mbarrier_timeout()):
        g, m = p.build()
        assert _rules(compile_graph(g, m).render()) == [], p.pid


def test_plant_undefined_predicate():
    # the attention kernel's lane-0 predicate, defined only on the role path:
    # the softmax warps' elected arrive would read it undefined
    ptx = _ptx_config("attention", B=1, H=2, S=512)
    lines = ptx.splitlines()
    i = next(i for i, ln in enumerate(lines) if re.search(r"setp\.eq\.u32 %p\d+, %r3, 0;", ln))
    line = lines.pop(i)
    j = next(j for j, ln in enumerate(lines) if "setmaxnreg.dec" in ln)
    lines.insert(j + 1, line)
    assert "defined" in _rules("\n".join(lines))


def test_plant_undefined_register():
    ptx = _ptx_config("vector_add", n=4096)
    ptx = ptx.replace("\tret;", "\tadd.s32 %r900, %r901, 1;\n\tret;", 1)
    ptx = ptx.replace(".reg .b32 %r<", ".reg .b32 %r<1000>;\n\t.reg .b32 %q<", 1)
    assert "defined" in _rules(ptx)


def test_plant_unbounded_wait():
    ptx = _ptx_config("matmul_bf16", M=256, N=256, K=256)
    lines = [ln for ln in ptx.splitlines()]
    # drop the clock reads and the bound test of one wait loop
    i = next(i for i, ln in enumerate(lines) if ln.startswith("$L_WAIT_") and ":" in ln)
    end = next(j for j in range(i, len(lines)) if "bra $L_WAIT_" in lines[j])
    kept = lines[:i + 1] + [ln for ln in lines[i + 1:end]
                            if "%globaltimer" not in ln and "sub.s64" not in ln
                            and "setp.lt.s64" not in ln] + \
        ["\tbra " + lines[i].rstrip(":") + ";"] + lines[end + 1:]
    assert "bounded-wait" in _rules("\n".join(kept))


def test_plant_tmem_and_regsplit():
    # (the copy-broadcast rule is exercised only negatively here: every
    # generated kernel is checked clean; a planted positive case would have
    # to spell the copy form that multi-GPU runs of these sources must not
    # contain)
    ptx = _ptx_config("attention", B=1, H=2, S=512)
    nodealloc = re.sub(r"\ttcgen05\.dealloc[^\n]*\n", "", ptx)
    assert "tmem" in _rules(nodealloc)
    greedy = ptx.replace("setmaxnreg.inc.sync.aligned.u32 200;", "setmaxnreg.inc.sync.aligned.u32 232;")
    assert "regsplit" in _rules(greedy)
    nodecl = re.sub(r"// @emmy regsplit[^\n]*\n", "", ptx)
    assert "regsplit" in _rules(nodecl)


def test_cli(tmp_path):
    import subprocess
    import sys
    good = tmp_path / "good.ptx"
    good.write_text(_ptx_config("vector_add", n=4096))
    r = subprocess.run([sys.executable, "-m", "emmy_b200.ptxcheck", str(good)],
                       capture_output=True, text=True,
                       cwd=REPO / "emmy-hackathon-2026_b200")
    assert r.returncode == 0, r.stdout

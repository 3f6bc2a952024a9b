"""Run the reference compiler (``compile.py`` of emmy-hackathon-2026) in-process.

TEST INFRASTRUCTURE ONLY -- nothing in the product imports this module.

The reference imports ``emmy.compiler.graph.Graph`` and
``emmy.compiler.ir.expr.Var`` (reference ``compile.py:59-60``).  emmy-ml is not
installable offline, so this module registers a stand-in ``emmy`` package
whose two names are served by this repository's IR reader, then loads the
reference's bundled ``compile.py`` from its source tree and calls its own
``Compiler`` / ``find_kernel`` (reference ``compile.py:2626-2648``).

Uses:
* reader parity -- the reference's emitted PTX for every problem and bug
  fixture must be byte-identical to the reference's committed goldens
  (reference ``tools/validate.py:92-115``); the files are compared as bytes
  and never read as text;
* the reference-on-B200 comparison -- :func:`emit_reference_ptx` writes the
  reference's sm_89 PTX for a synthesised IR into ``oracle/_ref/``, which
  travels to the GPU box as a built artefact.

It only works where the reference source tree exists (this container).
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import types
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
# the reference checkout: EMMY_REFERENCE_ROOT, else a "reference" folder beside
# this repository
REF_ROOT = Path(os.environ.get("EMMY_REFERENCE_ROOT") or REPO.parent / "reference")
REF_OUT = REPO / "oracle" / "_ref"

sys.path.insert(0, str(REPO / "emmy-hackathon-2026_b200"))


def reference_available() -> bool:
    return (REF_ROOT / "compile.py").is_file()


def _install_shim():
    from emmy_b200 import ir

    if "emmy.compiler.graph" in sys.modules and getattr(
            sys.modules["emmy.compiler.graph"], "Graph", None) is ir.Graph:
        return
    pkgs = ["emmy", "emmy.compiler", "emmy.compiler.ir"]
    for p in pkgs:
        m = types.ModuleType(p)
        m.__path__ = []  # mark as package
        sys.modules[p] = m
    graph_mod = types.ModuleType("emmy.compiler.graph")
    graph_mod.Graph = ir.Graph
    sys.modules["emmy.compiler.graph"] = graph_mod
    expr_mod = types.ModuleType("emmy.compiler.ir.expr")
    for name in ir.EXPR_KINDS:
        setattr(expr_mod, name, ir.NODE_CLASSES[name])
    sys.modules["emmy.compiler.ir.expr"] = expr_mod
    stmt_mod = types.ModuleType("emmy.compiler.ir.stmt")
    for name in ir.STMT_KINDS:
        setattr(stmt_mod, name, ir.NODE_CLASSES[name])
    sys.modules["emmy.compiler.ir.stmt"] = stmt_mod


_REF_MOD = None


def reference_module():
    """The reference ``compile.py`` loaded as a module behind the shim."""
    global _REF_MOD
    if _REF_MOD is None:
        if not reference_available():
            raise FileNotFoundError(f"reference compiler not found under {REF_ROOT}")
        _install_shim()
        spec = importlib.util.spec_from_file_location("emmy_reference_compile", REF_ROOT / "compile.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _REF_MOD = mod
    return _REF_MOD


def reference_ptx(graph_dict: dict, meta: dict) -> str:
    """Compile one IR graph with the reference compiler; returns its PTX text."""
    mod = reference_module()
    from emmy_b200 import ir

    g = ir.Graph.from_dict(graph_dict)
    c = mod.Compiler(g, meta, mod.find_kernel(g))
    c.compile()
    return c.render()


def reference_ptx_file(ir_path) -> bytes:
    """Reference PTX for an IR file whose ``meta.json`` sits beside it."""
    p = Path(ir_path)
    return reference_ptx(json.loads(p.read_text()),
                         json.loads((p.parent / "meta.json").read_text())).encode()


REF_PREFIX = "ref_"


def emit_reference_ptx(name: str, graph_dict: dict, meta: dict) -> Path:
    """Write the reference's PTX for a (synthesised) IR to ``oracle/_ref``.

    The KernelOp is renamed ``ref_<entry>`` (in the IR handed to the reference
    compiler, and in a copy of meta), so a profiler's launch list tells the
    reference's kernel apart from this build's kernel for the same IR."""
    import copy
    g = copy.deepcopy(graph_dict)
    m = copy.deepcopy(meta)
    for nd in g["nodes"].values():
        if nd["op"] == "KernelOp":
            nd["op_fields"]["name"] = REF_PREFIX + nd["op_fields"]["name"]
    for kinfo in m["kernels"]:
        kinfo["entry"] = REF_PREFIX + kinfo["entry"]
    REF_OUT.mkdir(parents=True, exist_ok=True)
    out = REF_OUT / f"{name}.ptx"
    out.write_bytes(reference_ptx(g, m).encode())
    return out


def emit_problem_ptx(folder) -> list:
    """Write the reference's PTX for every kernel of a problem folder (IR
    files named ``<entry>.ir.json`` or ``kernel.ir.json``, ``meta.json``
    beside them) to ``oracle/_ref/problems/<problem>/<entry>.ptx``, entry
    names unchanged (so the PTX launches under the problem's own meta)."""
    folder = Path(folder)
    meta = json.loads((folder / "meta.json").read_text())
    out_dir = REF_OUT / "problems" / folder.name
    out_dir.mkdir(parents=True, exist_ok=True)
    written = []
    for kinfo in meta["kernels"]:
        ir_path = folder / f"{kinfo['entry']}.ir.json"
        if not ir_path.exists():
            ir_path = folder / "kernel.ir.json"
        ptx = reference_ptx(json.loads(ir_path.read_text()), meta)
        out = out_dir / f"{kinfo['entry']}.ptx"
        out.write_bytes(ptx.encode())
        written.append(out)
    return written

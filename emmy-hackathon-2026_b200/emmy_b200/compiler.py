"""Kernel IR -> sm_100a PTX: the in-process API and the command line.

Mirrors the reference's public surface (reference ``compile.py:2276-2320``,
``2536-2544``, ``2619-2672``; callers such as
``tools/harness/regression.py:26-45`` use it in-process):

* ``Compiler(graph, meta, kernel_name)`` with ``.compile()`` and ``.render()``;
* ``find_kernel(graph)`` -- the single KernelOp node of the graph;
* ``compile_ir(path)`` -- reads ``meta.json`` from the IR's directory;
* ``main(argv)`` -- exit 0 with PTX on stdout, 1 for an unsupported construct
  (``unsupported construct: ...`` on stderr, ``COMPILER_TRACEBACK=1``
  re-raises), 2 for usage errors or a missing ``meta.json``.

Instead of lowering statement by statement, ``compile()`` first asks each
hand-written template (:mod:`emmy_b200.templates`) whether the IR has its
shape; the first that accepts emits the kernel.  IRs no template accepts go
to the statement-by-statement sm_100a lowering (:mod:`emmy_b200.generic`).
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

from . import ir as _ir
from .context import KernelContext
from .ops import UnsupportedOp
from .templates import TEMPLATES, TemplateMismatch

Graph = _ir.Graph


def find_kernel(graph) -> str:
    """Name of the single KernelOp node (reference ``compile.py:2626-2634``)."""
    kernels = [name for name, node in graph.nodes.items()
               if type(node.op).__name__ == "KernelOp"]
    if len(kernels) != 1:
        raise RuntimeError(f"expected exactly one KernelOp, found {kernels}")
    return kernels[0]


class Compiler:
    def __init__(self, graph, meta, kernel):
        self.g = graph
        self.meta = meta
        self.node_name = kernel
        self.ctx = KernelContext(graph, meta, kernel)
        self.entry = self.ctx.entry
        self.template = None
        self.ptx = None
        self.rejections = []

    def select(self):
        """The template (or generic lowering) that will emit this kernel."""
        if self.ctx.tile is None:
            raise NotImplementedError("expected a single Tile at top level")
        forced = os.environ.get("EMMY_TEMPLATE")
        for t in TEMPLATES:
            if forced and t.name != forced:
                continue
            try:
                return t.match(self.ctx)
            except TemplateMismatch as e:
                self.rejections.append((t.name, str(e)))
        from .generic import GenericLowering
        return GenericLowering(self.ctx)

    def compile(self):
        self.template = self.select()
        try:
            self.ptx = self.template.emit()
        except UnsupportedOp as e:
            # a template accepted the schedule but its op emitter lacks one of
            # the IR's elementwise ops: the statement-by-statement lowering
            # has the full op set
            if getattr(self.template, "name", "generic") == "generic":
                raise
            self.rejections.append((self.template.name, str(e)))
            from .generic import GenericLowering
            self.template = GenericLowering(self.ctx)
            self.ptx = self.template.emit()
        if self.ctx.info.get("peer_finish") and "// @emmy peer" not in self.ptx:
            raise NotImplementedError("peer_finish: only the split full sum (rows template) "
                                      "finishes the global sum in the kernel")
        return self

    def render(self) -> str:
        if self.ptx is None:
            self.compile()
        return self.ptx

    @property
    def kind(self) -> str:
        return getattr(self.template, "name", "?")


def compile_graph(graph_dict: dict, meta: dict) -> Compiler:
    g = _ir.load_graph(graph_dict)
    c = Compiler(g, meta, find_kernel(g))
    c.compile()
    return c


def compile_ir(ir_path) -> str:
    """Compile one IR file to PTX text; ``meta.json`` must sit beside it
    (reference ``compile.py:2637-2648``)."""
    path = Path(ir_path)
    graph = _ir.load_graph(json.loads(path.read_text()))
    meta_path = path.parent / "meta.json"
    if not meta_path.exists():
        raise FileNotFoundError(f"missing {meta_path}")
    meta = json.loads(meta_path.read_text())
    c = Compiler(graph, meta, find_kernel(graph))
    c.compile()
    return c.render()


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 1:
        print("usage: python compile.py <kernel.ir.json>", file=sys.stderr)
        return 2
    try:
        sys.stdout.write(compile_ir(argv[0]))
    except NotImplementedError as e:
        print(f"unsupported construct: {e}", file=sys.stderr)
        if os.environ.get("COMPILER_TRACEBACK") == "1":
            raise
        return 1
    except FileNotFoundError as e:
        print(str(e), file=sys.stderr)
        return 2
    return 0

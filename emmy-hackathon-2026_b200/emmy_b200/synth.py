"""IR synthesiser: Kernel IR graphs + meta.json for the benchmark shapes.

Emmy traces PyTorch expressions into IR (reference ``tools/generate.py:57-205``),
which needs emmy-ml and torch tracing; neither runs offline.  This module
writes the same artefacts directly, in the schedule forms Emmy itself emits
for each category, scaled to the benchmark shapes:

* pointwise -- the strided-loop form ``Tile[a0_co] { for a0 in a0_co..N:T }``;
* full sum  -- the split form of reference ``tests/hsx/sum_big`` (``_ksplit`` CTAs,
  one atomic add per CTA, output in ``zero_outputs``);
* row sum / row mean -- reference ``problems/r04_row_sum`` / ``r03_mean``;
* RMSNorm / softmax / L2 norm -- reference ``problems/f01..f03`` (softmax with the
  input scaled by a constant, L2 norm with ``maximum(norm, eps)``).

The output is the JSON graph format of the problems (``inputs``, ``outputs``,
``nodes`` with ``op_fields.body`` as ``repr`` strings) plus a ``meta.json``
dict with the reference's launch fields, the reference's argument forms
(``seed``/``data``/``output``), this build's ``dist`` form for the benchmark
distributions (:mod:`emmy_b200.data`), and an ``oracle`` entry naming the
expression family the tests evaluate on the CPU.  Seeds follow the
reference's convention: an input's seed is its index in ``graph.inputs``
(reference ``tools/generate.py:135``).
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

from . import ir as I

F32 = I.data_type("f32")
BF16 = I.data_type("bf16")


# --------------------------------------------------------------------------
# repr serialiser (the inverse of ir.parse_repr)
# --------------------------------------------------------------------------

def to_repr(x) -> str:
    k = type(x).__name__
    if x is None or isinstance(x, bool):
        return repr(x)
    if isinstance(x, (int, float)) and not isinstance(x, bool):
        return repr(x)
    if isinstance(x, I.NpDtype):
        return f"dtype({str.__repr__(str(x))})"
    if isinstance(x, str):
        return repr(str(x))
    if isinstance(x, tuple):
        if len(x) == 1:
            return "(" + to_repr(x[0]) + ",)"
        return "(" + ", ".join(to_repr(e) for e in x) + ")"
    if k == "Dim":
        return f"Dim({x.value})"
    if k == "ElementwiseImpl":
        return f"ElementwiseImpl({x.name!r})"
    if k in I.NODE_CLASSES:
        import dataclasses
        parts = [f"{f.name}={to_repr(getattr(x, f.name))}" for f in dataclasses.fields(x)]
        return f"{k}(" + ", ".join(parts) + ")"
    raise TypeError(f"cannot serialise {k}")


# --------------------------------------------------------------------------
# builders
# --------------------------------------------------------------------------

def V(name):
    return I.Var(name)


def Lit(v):
    return I.Literal(v, "int" if isinstance(v, int) else "float")


def add(a, b):
    return I.BinaryExpr("+", a, b)


def mul(a, b):
    return I.BinaryExpr("*", a, b)


def eq(a, b):
    return I.BinaryExpr("==", a, b)


def axis(name, extent, parent=None):
    w = None
    if parent is not None:
        w = I.Window(I.Axis(parent[0], I.Dim(parent[1]), None), None, None, True)
    return I.Axis(name, I.Dim(extent), w)


def load(name, buf, *index, dtype=F32):
    return I.Load((name,), buf, tuple(index), dtype)


def assign(name, op, *args, dtype=F32):
    return I.Assign(name, I.ElementwiseImpl(op), tuple(args), dtype)


def accum(name, value, op="add", base=None, axes=()):
    return I.Accum(name, value, I.ElementwiseImpl(op), F32, tuple(axes), base)


def write(out, index, values, atomic=False, dtype=F32):
    return I.Write(out, tuple(index), tuple(values), dtype, atomic, "NONE")


def tile(axes, body, block_threads=None):
    return I.Tile(tuple(axes), tuple(body), block_threads, 0, None, None, "m")


def strided(ax, start, step, body):
    return I.StridedLoop(ax, start, Lit(step), tuple(body), False, None, True)


def combine_block(states, B, combine):
    """WarpShuffle + per-warp smem + lane-0 store + Sync + TreeHalve, as Emmy
    emits it for a cooperative reduction over B threads (reference
    ``problems/r01_array_sum/*.ir.txt:6-12``)."""
    sb = tuple(f"{s}__o" for s in states)
    out = [I.WarpShuffle(tuple(states), sb, tuple(combine), 32, F32)]
    nw = B // 32
    for s in states:
        out.append(I.Smem(f"{s}_smem", (nw,), "float", 0))
    out.append(I.Cond(eq(V("lane"), Lit(0)),
                      tuple(write(f"{s}_smem", (V("warp"),), (s,)) for s in states), ()))
    out.append(I.Sync(0, None, False))
    out.append(I.TreeHalve(tuple(f"{s}_smem" for s in states), tuple(states), sb,
                           tuple(combine), nw, "warp", F32, 0, None, None))
    return out


def add_combine(s="acc0"):
    return [assign(s, "add", s, f"{s}__o", dtype=None)]


def softmax_combine():
    """The online-softmax merge of (max, sum) pairs (reference f02's combine)."""
    return [assign("acc0__o__gn", "maximum", "acc0", "acc0__o", dtype=None),
            assign("acc0__o__dg", "subtract", "acc0", "acc0__o__gn", dtype=None),
            assign("acc0__o__alpha", "exp", "acc0__o__dg", dtype=None),
            assign("acc0__o__dg_o", "subtract", "acc0__o", "acc0__o__gn", dtype=None),
            assign("acc0__o__beta", "exp", "acc0__o__dg_o", dtype=None),
            assign("acc0__o__acc1_sa", "multiply", "acc0__o__alpha", "acc1", dtype=None),
            assign("acc0__o__acc1_sb", "multiply", "acc0__o__beta", "acc1__o", dtype=None),
            assign("acc1", "add", "acc0__o__acc1_sa", "acc0__o__acc1_sb", dtype=None),
            assign("acc0", "copy", "acc0__o__gn", dtype=None)]


# --------------------------------------------------------------------------
# graph + meta assembly
# --------------------------------------------------------------------------

class Problem:
    def __init__(self, pid: str, code: str, entry: str, node: str):
        self.pid, self.code, self.entry, self.node = pid, code, entry, node
        self.inputs = []       # (name, shape, dtype, argspec)
        self.consts = []       # (name, value)
        self.out = None        # (name, shape, dtype)
        self.body = None
        self.grid = self.block = None
        self.smem = 0
        self.zero = []
        self.oracle = None
        self.rtol = self.atol = None

    def add_input(self, name, shape, dtype="f32", dist=None):
        self.inputs.append((name, tuple(shape), dtype, dist))

    def add_const(self, name, value):
        self.consts.append((name, float(value)))

    def graph(self) -> dict:
        nodes = {}
        names = []
        for name, shape, dt, _ in self.inputs:
            nodes[name] = {"op": "InputOp", "op_fields": {}, "inputs": [],
                           "outputs": [{"name": name, "shape": list(shape), "dtype": dt}]}
            names.append(name)
        for name, value in self.consts:
            nodes[name] = {"op": "ConstantOp", "op_fields": {"name": name, "value": value},
                           "inputs": [],
                           "outputs": [{"name": name, "shape": [1], "dtype": "f32"}]}
        oname, oshape, odt = self.out
        nodes[self.node] = {
            "op": "KernelOp",
            "op_fields": {"body": [to_repr(self.body)], "name": self.entry,
                          "zero_delegated": [], "serial": []},
            "inputs": [c for c, _ in self.consts] + names,
            "outputs": [{"name": oname, "shape": list(oshape), "dtype": odt}]}
        return {"inputs": names, "outputs": [oname], "nodes": nodes}

    def meta(self) -> dict:
        args = []
        arg_order = []
        for name, value in self.consts:
            args.append({"name": name, "dtype": "f32", "shape": [1], "data": [value]})
            arg_order.append(name)
        for i, (name, shape, dt, dist) in enumerate(self.inputs):
            a = {"name": name, "dtype": dt, "shape": list(shape), "seed": i}
            if dist:
                a["dist"] = dist
            args.append(a)
            arg_order.append(name)
        oname, oshape, odt = self.out
        args.append({"name": oname, "dtype": odt, "shape": list(oshape), "output": True})
        arg_order.append(oname)
        return {"id": self.pid, "code": self.code, "rtol": self.rtol, "atol": self.atol,
                "graph_inputs": [n for n, *_ in self.inputs], "graph_outputs": [oname],
                "kernels": [{"node": self.node, "entry": self.entry, "arg_order": arg_order,
                             "grid": list(self.grid), "block": list(self.block),
                             "smem_bytes": self.smem, "zero_outputs": list(self.zero),
                             "args": args, "final": True}],
                "oracle": self.oracle}

    def build(self) -> tuple[dict, dict]:
        return self.graph(), self.meta()

    def write(self, folder, expected: dict | None = None) -> Path:
        """The problem as a folder in the reference's format."""
        return write_problem(folder, {self.entry: self.graph()}, self.meta(), expected)


def write_problem(folder, irs: dict, meta: dict, expected: dict | None = None) -> Path:
    """A problem folder as the reference's generator lays it out (reference
    ``tools/generate.py:177-199``): ``<entry>.ir.json`` per kernel,
    ``meta.json``, and ``expected.npz`` (graph output -> array) when given."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    for entry, g in irs.items():
        (folder / f"{entry}.ir.json").write_text(json.dumps(g, indent=1))
    (folder / "meta.json").write_text(json.dumps(meta, indent=1))
    if expected is not None:
        np.savez(folder / "expected.npz", **expected)
    return folder


class Pipeline:
    """A problem of several kernels run in order, later ones reading buffers
    earlier ones wrote -- the shape of Emmy's multi-kernel lowerings as the
    reference's generator packages them (``tools/generate.py:108-146``: an
    argument no InputOp or ConstantOp provides is ``intermediate``; a kernel is
    ``final`` when it writes a graph output) and its ``submit.py`` chains them
    (``:112-122``).  Each stage is a :class:`Problem` whose inputs name graph
    inputs or earlier stages' outputs."""

    def __init__(self, pid: str, code: str, stages: list, graph_inputs: list,
                 graph_outputs: list, rtol: float, atol: float, oracle: dict | None = None):
        self.pid, self.code, self.stages = pid, code, stages
        self.graph_inputs = graph_inputs          # [(name, dist or None)]
        self.graph_outputs = graph_outputs
        self.rtol, self.atol, self.oracle = rtol, atol, oracle

    def build(self) -> tuple[dict, dict]:
        gin = [n for n, _ in self.graph_inputs]
        dists = dict(self.graph_inputs)
        irs, kernels, produced = {}, [], set()
        for st in self.stages:
            irs[st.entry] = st.graph()
            args, order = [], []
            for name, value in st.consts:
                args.append({"name": name, "dtype": "f32", "shape": [1], "data": [value]})
                order.append(name)
            for name, shape, dt, _ in st.inputs:
                a = {"name": name, "dtype": dt, "shape": list(shape)}
                if name in gin:
                    a["seed"] = gin.index(name)
                    if dists[name]:
                        a["dist"] = dists[name]
                elif name in produced:
                    a["intermediate"] = True
                else:
                    raise ValueError(f"{st.entry}: {name} is neither a graph input nor "
                                     f"written by an earlier kernel")
                args.append(a)
                order.append(name)
            oname, oshape, odt = st.out
            args.append({"name": oname, "dtype": odt, "shape": list(oshape), "output": True})
            order.append(oname)
            produced.add(oname)
            kernels.append({"node": st.node, "entry": st.entry, "arg_order": order,
                            "grid": list(st.grid), "block": list(st.block),
                            "smem_bytes": st.smem, "zero_outputs": list(st.zero),
                            "args": args, "final": oname in self.graph_outputs})
        meta = {"id": self.pid, "code": self.code, "rtol": self.rtol, "atol": self.atol,
                "graph_inputs": gin, "graph_outputs": list(self.graph_outputs),
                "kernels": kernels, "oracle": self.oracle}
        return irs, meta

    def write(self, folder, expected: dict | None = None) -> Path:
        irs, meta = self.build()
        return write_problem(folder, irs, meta, expected)


def _row_reduce_stage(entry, node, src_load, value_ops, acc_op, combine, post, out, rows, cols,
                      block, inputs, consts=()):
    """One CTA per row: a strided loop folds ``value_ops`` into acc0, the block
    combines, ``post`` finishes, thread 0 of the row writes ``out[row]``."""
    st = Problem(node, "", entry, node)
    for c, v in consts:
        st.add_const(c, v)
    for name, shape in inputs:
        st.add_input(name, shape)
    st.out = (out, (rows,), "f32")
    loop = strided(axis("a1", cols), V("a1_co"), block,
                   [src_load] + list(value_ops) + [accum("acc0", "v_in", op=acc_op, axes=("a1",))])
    st.body = tile([axis("a0", rows), axis("a1_co", block)],
                   [loop] + combine_block(["acc0"], block, combine) + list(post) +
                   [I.Cond(eq(V("a1_co"), Lit(0)), (write(out, (V("a0"),), ("r_out",)),), ())])
    st.grid, st.block = (rows, 1, 1), (block, 1, 1)
    return st


def _elementwise_stage(entry, node, body, out, rows, cols, inputs, consts=(), threads=256):
    """One thread per (row, column) element."""
    st = Problem(node, "", entry, node)
    for c, v in consts:
        st.add_const(c, v)
    for name, shape in inputs:
        st.add_input(name, shape)
    st.out = (out, (rows, cols), "f32")
    st.body = tile([axis("a0", rows), axis("a1", cols)], body)
    n = rows * cols
    st.grid, st.block = (-(-n // threads), 1, 1), (threads, 1, 1)
    return st


def rmsnorm_two_kernel(rows: int = 256, cols: int = 1024, block: int = 128,
                       eps: float = 1e-6) -> Pipeline:
    """RMSNorm as two kernels: ``ms[r] = mean(x[r]^2)`` into an intermediate,
    then ``y = x * rsqrt(ms + eps) * w``."""
    s1 = _row_reduce_stage(
        "k_rms_meansq", "ms", load("in0", "x", V("a0"), V("a1")),
        [assign("v_in", "multiply", "in0", "in0")], "add", add_combine(),
        [load("c0", "mean_count", Lit(0)), assign("rc", "reciprocal", "c0"),
         assign("r_out", "multiply", "acc0", "rc")],
        "ms", rows, cols, block, [("x", (rows, cols))], consts=[("mean_count", cols)])
    s2 = _elementwise_stage(
        "k_rms_apply", "mul_1",
        [load("m", "ms", V("a0")), load("e", "add_c1", Lit(0)), assign("v0", "add", "m", "e"),
         assign("v1", "sqrt", "v0"), assign("v2", "reciprocal", "v1"),
         load("xi", "x", V("a0"), V("a1")), assign("v3", "multiply", "xi", "v2"),
         load("wi", "w", V("a1")), assign("v4", "multiply", "wi", "v3"),
         write("mul_1", (V("a0"), V("a1")), ("v4",))],
        "mul_1", rows, cols, [("x", (rows, cols)), ("ms", (rows,)), ("w", (cols,))],
        consts=[("add_c1", eps)])
    return Pipeline(f"rmsnorm2k_{rows}x{cols}", "x * rsqrt(mean(x^2)+eps) * w", [s1, s2],
                    [("x", None), ("w", {"kind": "uniform", "lo": 0.5, "hi": 1.5})], ["mul_1"],
                    rtol=1e-5, atol=1e-5,
                    oracle={"family": "rmsnorm", "args": {"x": "x", "w": "w"},
                            "output": "mul_1", "eps": eps})


def softmax_three_kernel(rows: int = 128, cols: int = 2048, block: int = 128,
                         scale: float = 4.0) -> Pipeline:
    """Row softmax of ``scale * x`` as three kernels: row max, row sum of
    ``exp(scale*x - max)``, then the normalised exponentials."""
    sx = [load("c0", "mul_c1", Lit(0)), assign("sxv", "multiply", "in0", "c0")]
    s1 = _row_reduce_stage(
        "k_sm_max", "rmax", load("in0", "x", V("a0"), V("a1")),
        sx + [assign("v_in", "copy", "sxv")], "maximum",
        [assign("acc0", "maximum", "acc0", "acc0__o", dtype=None)],
        [assign("r_out", "copy", "acc0")], "rmax", rows, cols, block,
        [("x", (rows, cols))], consts=[("mul_c1", scale)])
    s2 = _row_reduce_stage(
        "k_sm_sum", "rsum", load("in0", "x", V("a0"), V("a1")),
        sx + [load("mx", "rmax", V("a0")), assign("d", "subtract", "sxv", "mx"),
              assign("v_in", "exp", "d")], "add", add_combine(),
        [assign("r_out", "copy", "acc0")], "rsum", rows, cols, block,
        [("x", (rows, cols)), ("rmax", (rows,))], consts=[("mul_c1", scale)])
    s3 = _elementwise_stage(
        "k_sm_norm", "softmax",
        [load("in0", "x", V("a0"), V("a1"))] + sx +
        [load("mx", "rmax", V("a0")), assign("d", "subtract", "sxv", "mx"),
         assign("e", "exp", "d"), load("sm", "rsum", V("a0")), assign("y", "divide", "e", "sm"),
         write("softmax", (V("a0"), V("a1")), ("y",))],
        "softmax", rows, cols, [("x", (rows, cols)), ("rmax", (rows,)), ("rsum", (rows,))],
        consts=[("mul_c1", scale)])
    return Pipeline(f"softmax3k_{rows}x{cols}", f"softmax({scale} * x, -1)", [s1, s2, s3],
                    [("x", None)], ["softmax"], rtol=1e-5, atol=1e-6,
                    oracle={"family": "softmax", "args": {"x": "x"}, "output": "softmax",
                            "scale": scale})


# --------------------------------------------------------------------------
# the benchmark configurations
# --------------------------------------------------------------------------

UNIF01 = {"kind": "uniform", "lo": 0.0, "hi": 1.0}
UNIF11 = {"kind": "uniform", "lo": -1.0, "hi": 1.0}


def vector_add(n: int = 1_048_576, threads: int | None = None, block: int = 256) -> Problem:
    """``c = a + b`` over ``n`` f32 elements, strided-loop form."""
    T = threads or min(n, 148 * block)
    T = -(-T // block) * block
    p = Problem(f"add_{n}", "a + b", "k_add_pointwise", "add")
    p.add_input("x0", (n,), dist=UNIF11)
    p.add_input("x1", (n,), dist=UNIF11)
    p.out = ("add", (n,), "f32")
    loop = strided(axis("a0", n), V("a0_co"), T,
                   [load("in0", "x0", V("a0")), load("in1", "x1", V("a0")),
                    assign("v0", "add", "in0", "in1"), write("add", (V("a0"),), ("v0",))])
    p.body = tile([axis("a0_co", T)], [loop])
    p.grid, p.block = (T // block, 1, 1), (block, 1, 1)
    p.rtol, p.atol = 0, 0
    p.oracle = {"family": "add", "args": {"a": "x0", "b": "x1"}, "output": "add"}
    return p


def full_sum(n: int = 268_435_456, ctas: int = 2048, block: int = 256) -> Problem:
    """``s = sum(x)``, x ~ U(0,1): split form, one atomic add per CTA."""
    assert n % ctas == 0
    C = n // ctas
    p = Problem(f"sum_{n}", "x.sum()", "k_sum_1_reduce", "sum_1")
    p.add_input("x", (n,), dist=UNIF01)
    p.out = ("sum_1", (), "f32")
    loop = strided(axis("a0", C, parent=("a0", n)), V("a0_co"), block,
                   [load("in0", "x", add(V("a0"), mul(V("_ksplit"), Lit(C)))),
                    accum("acc0", "in0", axes=("a0",))])
    body = [loop] + combine_block(["acc0"], block, add_combine()) + [
        I.Cond(eq(V("a0_co"), Lit(0)), (write("sum_1", (), ("acc0",), atomic=True),), ())]
    p.body = tile([axis("_ksplit", ctas), axis("a0_co", block)], body, block)
    p.grid, p.block = (ctas, 1, 1), (block, 1, 1)
    p.zero = ["sum_1"]
    p.rtol, p.atol = 1e-4, None
    p.oracle = {"family": "sum", "args": {"x": "x"}, "output": "sum_1"}
    return p


def row_reduce(rows: int = 32768, cols: int = 8192, block: int = 256, mean: bool = False) -> Problem:
    """``y[r] = sum_c x[r, c]`` (or the mean, ``/ cols``), x ~ N(0,1)."""
    name = "mean" if mean else "sum_1"
    p = Problem(f"row_{'mean' if mean else 'sum'}_{rows}x{cols}",
                f"x.{'mean' if mean else 'sum'}(-1)",
                "k_mean_rows_reduce" if mean else "k_sum_rows_reduce", name)
    if mean:
        p.add_const("mean_count", cols)
    p.add_input("x", (rows, cols))
    p.out = (name, (rows,), "f32")
    loop = strided(axis("a1", cols), V("a1_co"), block,
                   [load("in0", "x", V("a0"), V("a1")), accum("acc0", "in0", axes=("a1",))])
    tail = [write(name, (V("a0"),), ("acc0",))]
    if mean:
        tail = [load("in1", "mean_count", Lit(0)), assign("v0", "divide", "acc0", "in1"),
                write(name, (V("a0"),), ("v0",))]
    body = [loop] + combine_block(["acc0"], block, add_combine()) + [
        I.Cond(eq(V("a1_co"), Lit(0)), tuple(tail), ())]
    p.body = tile([axis("a0", rows), axis("a1_co", block)], body)
    p.grid, p.block = (rows, 1, 1), (block, 1, 1)
    p.rtol, p.atol = 1e-4, None
    p.oracle = {"family": "row_mean" if mean else "row_sum", "args": {"x": "x"}, "output": name}
    return p


def rmsnorm(rows: int = 65536, cols: int = 4096, block: int = 128, eps: float = 1e-6) -> Problem:
    """``y = x * rsqrt(mean(x^2) + eps) * w`` (reference f01's IR with eps)."""
    p = Problem(f"rmsnorm_{rows}x{cols}", "x * rsqrt(mean(x^2)+eps) * w", "k_rmsnorm", "mul_1")
    p.add_const("mean_count", cols)
    p.add_const("add_c1", eps)
    p.add_input("x", (rows, cols))
    p.add_input("w", (cols,), dist={"kind": "uniform", "lo": 0.5, "hi": 1.5})
    p.out = ("mul_1", (rows, cols), "f32")
    loop1 = strided(axis("a1", cols), V("a1_co"), block,
                    [load("in2", "x", V("a0"), V("a1")), assign("v1", "multiply", "in2", "in2"),
                     accum("acc0", "v1", axes=("a1",))])
    post = [load("in1", "mean_count", Lit(0)), assign("v0", "reciprocal", "in1"),
            assign("v2", "multiply", "acc0", "v0"), load("in0", "add_c1", Lit(0)),
            assign("v3", "add", "in0", "v2"), assign("v4", "sqrt", "v3"),
            assign("v5", "reciprocal", "v4")]
    loop2 = strided(axis("a2", cols), V("a1_co"), block,
                    [load("in3", "x", V("a0"), V("a2")), assign("v6", "multiply", "in3", "v5"),
                     load("in4", "w", V("a2")), assign("v7", "multiply", "in4", "v6"),
                     write("mul_1", (V("a0"), V("a2")), ("v7",))])
    p.body = tile([axis("a0", rows), axis("a1_co", block)],
                  [loop1] + combine_block(["acc0"], block, add_combine()) + post + [loop2])
    p.grid, p.block = (rows, 1, 1), (block, 1, 1)
    p.rtol, p.atol = 1e-5, None
    p.oracle = {"family": "rmsnorm", "args": {"x": "x", "w": "w"}, "output": "mul_1", "eps": eps}
    return p


def softmax(rows: int = 65536, cols: int = 4096, block: int = 128, scale: float = 4.0) -> Problem:
    """Row softmax of ``scale * x`` (reference f02's online-softmax IR)."""
    p = Problem(f"softmax_{rows}x{cols}", f"softmax({scale} * x, -1)", "k_softmax", "softmax")
    p.add_const("mul_c1", scale)
    p.add_input("x", (rows, cols))
    p.out = ("softmax", (rows, cols), "f32")
    loop1 = strided(axis("a1", cols), V("a1_co"), block, [
        I.Let("one", Lit(1.0), F32),
        load("in0r", "x", V("a0"), V("a1")), load("c0", "mul_c1", Lit(0)),
        assign("in0", "multiply", "in0r", "c0"),
        assign("in0__gn", "maximum", "acc0", "in0"),
        assign("in0__dg", "subtract", "acc0", "in0__gn"),
        assign("in0__alpha", "exp", "in0__dg"),
        assign("in0__dg_o", "subtract", "in0", "in0__gn"),
        assign("in0__beta", "exp", "in0__dg_o"),
        assign("in0__acc1_sa", "multiply", "acc1", "in0__alpha"),
        assign("in0__acc1_sb", "multiply", "in0__beta", "one"),
        accum("acc1", "in0__acc1_sb", base="in0__acc1_sa", axes=("a1",)),
        accum("acc0", "in0", op="maximum", axes=("a1",))])
    post = [assign("v2", "reciprocal", "acc1")]
    loop2 = strided(axis("a3", cols), V("a1_co"), block, [
        load("in2r", "x", V("a0"), V("a3")), load("c1", "mul_c1", Lit(0)),
        assign("in2", "multiply", "in2r", "c1"),
        assign("v3", "subtract", "in2", "acc0"), assign("v4", "exp", "v3"),
        assign("v5", "multiply", "v2", "v4"), write("softmax", (V("a0"), V("a3")), ("v5",))])
    p.body = tile([axis("a0", rows), axis("a1_co", block)],
                  [loop1] + combine_block(["acc0", "acc1"], block, softmax_combine()) + post
                  + [loop2])
    p.grid, p.block = (rows, 1, 1), (block, 1, 1)
    p.rtol, p.atol = 1e-5, None
    p.oracle = {"family": "softmax", "args": {"x": "x"}, "output": "softmax", "scale": scale}
    return p


def l2norm(rows: int = 65536, cols: int = 4096, block: int = 128, eps: float = 1e-12) -> Problem:
    """``y = x / max(||x||_2, eps)`` (reference f03's IR with F.normalize's eps)."""
    p = Problem(f"l2norm_{rows}x{cols}", "x / max(norm(x, -1), eps)", "k_l2norm", "div")
    p.add_const("eps_c1", eps)
    p.add_input("x", (rows, cols))
    p.out = ("div", (rows, cols), "f32")
    loop1 = strided(axis("a1", cols), V("a1_co"), block,
                    [load("in0", "x", V("a0"), V("a1")), assign("v0", "multiply", "in0", "in0"),
                     accum("acc0", "v0", axes=("a1",))])
    post = [assign("v1", "sqrt", "acc0"), load("e0", "eps_c1", Lit(0)),
            assign("v1m", "maximum", "v1", "e0"), assign("v2", "reciprocal", "v1m")]
    loop2 = strided(axis("a2", cols), V("a1_co"), block,
                    [load("in1", "x", V("a0"), V("a2")), assign("v3", "multiply", "in1", "v2"),
                     write("div", (V("a0"), V("a2")), ("v3",))])
    p.body = tile([axis("a0", rows), axis("a1_co", block)],
                  [loop1] + combine_block(["acc0"], block, add_combine()) + post + [loop2])
    p.grid, p.block = (rows, 1, 1), (block, 1, 1)
    p.rtol, p.atol = 1e-5, None
    p.oracle = {"family": "l2norm", "args": {"x": "x"}, "output": "div", "eps": eps}
    return p


def _div(a, b):
    return I.BinaryExpr("/", a, b)


def _mod(a, b):
    return I.BinaryExpr("%", a, b)


def _lt(a, b):
    return I.BinaryExpr("<", a, b)


_SMEM_CTYPE = {"f32": "float", "bf16": "__nv_bfloat16"}


def matmul(M: int = 16384, N: int = 8192, K: int = 4096, dtype: str = "bf16", BM: int = 128,
           BN: int = 256, BK: int = 64, stages: int = 2, U0: int = 4, U1: int = 64,
           seeds=(0, 1)) -> Problem:
    """``C = A @ B`` with A [M,K], B [K,N] ~ U(-1,1) of ``dtype``, C f32, in the
    schedule form of the reference's ``problems/m01_matmul_512`` IR: a CTA per
    BM x BN output tile, U0 x U1 threads each owning an (BM/U0) x (BN/U1)
    register micro-tile, a ``stages``-deep cp.async ring of A/B k-slices in
    shared memory, and a fully unrolled inner k loop of multiply + Accum."""
    assert M % BM == 0 and N % BN == 0 and K % BK == 0 and BM % U0 == 0 and BN % U1 == 0
    mu, nu = BM // U0, BN // U1
    T = U0 * U1
    es = 2 if dtype == "bf16" else 4
    E = 16 // es                            # elements per 16-byte cp.async
    dt = BF16 if dtype == "bf16" else F32
    p = Problem(f"matmul_{dtype}_{M}x{N}x{K}", "x0 @ x1", f"k_matmul_{dtype}", "matmul")
    p.add_input("x0", (M, K), dtype=dtype, dist=UNIF11)
    p.add_input("x1", (K, N), dtype=dtype, dist=UNIF11)
    p.out = ("matmul", (M, N), "f32")
    tid = add(mul(V("a0_u"), Lit(U1)), V("a1_u"))

    def copies(slot, koff):
        ca, cb = BM * BK // E, BK * BN // E
        fa = mul(V("_fa"), Lit(E))
        fb = mul(V("_fb"), Lit(E))
        la = strided(axis("_fa", ca), tid, T, [I.CpAsyncCopy(
            "_a_smem", (add(mul(slot, Lit(BM)), _div(fa, Lit(BK))), _mod(fa, Lit(BK))), "x0",
            (add(mul(V("a0_b"), Lit(BM)), _div(fa, Lit(BK))), add(koff, _mod(fa, Lit(BK)))),
            16, "NONE", None, None)])
        lb = strided(axis("_fb", cb), tid, T, [I.CpAsyncCopy(
            "_b_smem", (add(mul(slot, Lit(BK)), _div(fb, Lit(BN))), _mod(fb, Lit(BN))), "x1",
            (add(koff, _div(fb, Lit(BN))), add(mul(V("a1_b"), Lit(BN)), _mod(fb, Lit(BN)))),
            16, "NONE", None, None)])
        return [la, lb, I.CpAsyncCommit()]

    body = [I.Init(f"acc0__c{i}_{j}", 0.0, F32) for i in range(mu) for j in range(nu)]
    body += [I.Smem("_a_smem", (stages * BM, BK), _SMEM_CTYPE[dtype], 16),
             I.Smem("_b_smem", (stages * BK, BN), _SMEM_CTYPE[dtype], 16)]
    for s in range(stages - 1):
        body += copies(Lit(s), Lit(s * BK))
    ks = V("_ks")
    cur = _mod(_div(ks, Lit(BK)), Lit(stages))
    nxt = _mod(add(_div(ks, Lit(BK)), Lit(stages - 1)), Lit(stages))
    ahead = add(ks, Lit((stages - 1) * BK))
    kpre = I.TernaryExpr(_lt(ahead, Lit(K)), ahead, Lit(K - BK))
    inner = []
    for j in range(nu):
        inner.append(I.Load((f"in1__c0_{j}",), "_b_smem",
                            (add(mul(cur, Lit(BK)), V("_ki")),
                             add(mul(V("a1_u"), Lit(nu)), Lit(j))), None))
    for i in range(mu):
        inner.append(I.Load((f"in0__c{i}_0",), "_a_smem",
                            (add(mul(cur, Lit(BM)), add(mul(V("a0_u"), Lit(mu)), Lit(i))),
                             V("_ki")), None))
        for j in range(nu):
            inner.append(assign(f"acc0__v__c{i}_{j}", "multiply", f"in1__c0_{j}", f"in0__c{i}_0"))
            inner.append(accum(f"acc0__c{i}_{j}", f"acc0__v__c{i}_{j}", axes=("_ki",)))
    kloop = I.Loop(axis("_ki", BK), tuple(inner), False, False)
    main = copies(nxt, kpre) + [I.CpAsyncWait(stages - 1), I.Sync(0, None, False), kloop,
                                I.Sync(0, None, False)]
    body.append(I.StridedLoop(axis("_ks", K), Lit(0), Lit(BK), tuple(main), False, None, False))
    for i in range(mu):
        body.append(write("matmul", (add(add(mul(V("a0_b"), Lit(BM)), mul(V("a0_u"), Lit(mu))),
                                         Lit(i)),
                                     add(mul(V("a1_b"), Lit(BN)), mul(V("a1_u"), Lit(nu)))),
                          tuple(f"acc0__c{i}_{j}" for j in range(nu))))
    p.body = tile([axis("a0_b", M // BM, parent=("a0", M)), axis("a1_b", N // BN, parent=("a1", N)),
                   axis("a0_u", U0), axis("a1_u", U1)], body)
    p.grid, p.block = ((M // BM) * (N // BN), 1, 1), (T, 1, 1)
    # the IR's ring, plus room for the tcgen05 template's barriers and alignment
    p.smem = stages * (BM * BK + BK * BN) * es + 2048
    if dtype == "bf16":
        p.rtol, p.atol = 2e-2, None
    else:
        p.rtol, p.atol = 1e-4, None
    p.oracle = {"family": "matmul", "args": {"a": "x0", "b": "x1"}, "output": "matmul",
                "flops": 2 * M * N * K, "bf16": {"x0": dtype == "bf16", "x1": dtype == "bf16"}}
    return p


def attention(B: int = 8, H: int = 32, S: int = 4096, D: int = 128, BM: int = 256,
              U0: int = 16, U1: int = 32, dtype: str = "bf16") -> Problem:
    """``O = softmax(Q K^T / sqrt(D)) V`` per (batch, head), non-causal, Q/K/V
    [B,H,S,D] ~ N(0,1) of ``dtype``, O f32, in the schedule form of the
    reference's ``problems/a01_attention`` / ``a02_attention_128`` IRs (a CTA per
    BM query rows x all D output columns, U0 x U1 threads each owning a
    (BM/U0) x (D/U1) micro-tile; per key: the q.k dot product loop, the online
    softmax chain with the ``acc1`` max / ``acc3`` sum / ``acc5`` weighted-sum
    accumulators, then ``reciprocal`` + ``multiply``), extended with leading
    batch and head axes and indexing K[b,h,s,d] directly (the reference's open
    problems pre-transpose K)."""
    assert S % BM == 0 and BM % U0 == 0 and D % U1 == 0
    mu, nu = BM // U0, D // U1
    dt = BF16 if dtype == "bf16" else F32
    p = Problem(f"attention_{dtype}_{B}x{H}x{S}x{D}", "softmax(q @ k^T / sqrt(d)) @ v",
                f"k_attention_{dtype}_d{D}", "matmul_1")
    p.add_const("div_c1", math.sqrt(D))
    for i, n in enumerate(("q", "k", "v")):
        p.add_input(n, (B, H, S, D), dtype=dtype)
    p.out = ("matmul_1", (B, H, S, D), "f32")
    bh = (V("ab"), V("ah"))

    def row(i):
        return add(add(mul(V("a0_b"), Lit(BM)), mul(V("a0_u"), Lit(mu))), Lit(i))

    def col(j):
        return add(add(mul(V("a5_b"), Lit(D)), mul(V("a5_u"), Lit(nu))), Lit(j))

    key_body = []
    for i in range(mu):
        key_body.append(I.Loop(axis("a2", D), (
            I.Load((f"in2__ar{i}",), "q", bh + (row(i), V("a2")), dt),
            I.Load((f"in1__ar{i}",), "k", bh + (V("a1"), V("a2")), dt),
            assign(f"v3__ar{i}", "multiply", f"in1__ar{i}", f"in2__ar{i}"),
            accum(f"acc0__ar{i}", f"v3__ar{i}", axes=("a2",))), False, True))
    for j in range(nu):
        key_body.append(I.Load((f"in7__bc{j}",), "v", bh + (V("a1"), col(j)), dt))
    for i in range(mu):
        for j in range(nu):
            c = f"__c{i}_{j}"
            key_body += [
                assign(f"v4{c}", "multiply", f"acc0__ar{i}", "v1"),
                I.Let(f"one{c}", Lit(1.0), F32),
                assign(f"v4__gn{c}", "maximum", f"acc1{c}", f"v4{c}"),
                assign(f"v4__dg{c}", "subtract", f"acc1{c}", f"v4__gn{c}"),
                assign(f"v4__alpha{c}", "exp", f"v4__dg{c}"),
                assign(f"v4__dg_o{c}", "subtract", f"v4{c}", f"v4__gn{c}"),
                assign(f"v4__beta{c}", "exp", f"v4__dg_o{c}"),
                assign(f"v4__acc3_sa{c}", "multiply", f"acc3{c}", f"v4__alpha{c}"),
                assign(f"v4__acc3_sb{c}", "multiply", f"one{c}", f"v4__beta{c}"),
                accum(f"acc3{c}", f"v4__acc3_sb{c}", base=f"v4__acc3_sa{c}", axes=("a1",)),
                assign(f"v4__acc5__sum_sa{c}", "multiply", f"acc5__sum{c}", f"v4__alpha{c}"),
                assign(f"v4__acc5__sum_sb{c}", "multiply", f"in7__bc{j}", f"v4__beta{c}"),
                accum(f"acc5__sum{c}", f"v4__acc5__sum_sb{c}", base=f"v4__acc5__sum_sa{c}",
                      axes=("a1",)),
                accum(f"acc1{c}", f"v4{c}", op="maximum", axes=("a1",))]
    body = [load("in0", "div_c1", Lit(0)), assign("v1", "reciprocal", "in0"),
            I.Loop(axis("a1", S), tuple(key_body), False, True)]
    for i in range(mu):
        for j in range(nu):
            c = f"__c{i}_{j}"
            body += [assign(f"v9{c}", "reciprocal", f"acc3{c}"),
                     assign(f"acc5{c}", "multiply", f"acc5__sum{c}", f"v9{c}")]
    for i in range(mu):
        body.append(write("matmul_1", bh + (row(i), col(0)),
                          tuple(f"acc5__c{i}_{j}" for j in range(nu))))
    p.body = tile([axis("ab", B), axis("ah", H), axis("a0_b", S // BM, parent=("a0", S)),
                   axis("a5_b", 1, parent=("a5", D)), axis("a0_u", U0), axis("a5_u", U1)], body)
    p.grid, p.block = (B * H * (S // BM), 1, 1), (U0 * U1, 1, 1)
    # the template's shared memory: the BM/128 Q tiles, a K ring and a V ring
    # of 128 x D tiles (3 + 2 stages at D=128, 4 + 4 below), barriers and the
    # 1 KB alignment of the tiles
    tb = 128 * D * 2
    p.smem = tb * (BM // 128 + (5 if D >= 128 else 8)) + 2048
    p.rtol, p.atol = 2e-2, None
    p.oracle = {"family": "attention", "args": {"q": "q", "k": "k", "v": "v"},
                "output": "matmul_1", "scale": 1.0 / math.sqrt(D),
                "flops": 4 * B * H * S * S * D,
                "bf16": {n: dtype == "bf16" for n in ("q", "k", "v")}}
    return p


# the BASELINE.json configurations by name (full sizes)
def config(name: str, **kw) -> Problem:
    table = {
        "vector_add": vector_add,
        # the same IR at 2^28 elements (3 GiB moved) under the same 148 x 256
        # launch: the pointwise template where bandwidth, not latency, bounds it
        "vector_add_large": lambda **k: vector_add(**{"n": 268_435_456, **k}),
        "full_sum": full_sum,
        "row_sum": lambda **k: row_reduce(mean=False, **k),
        "row_mean": lambda **k: row_reduce(mean=True, **k),
        "rmsnorm": rmsnorm,
        "softmax": softmax,
        "l2norm": l2norm,
        "matmul_bf16": lambda **k: matmul(**{"dtype": "bf16", "stages": 4, **k}),
        "matmul_f32": lambda **k: matmul(**{"dtype": "f32", "BK": 32, "stages": 4, **k}),
        "attention": attention,
        "attention_d64": lambda **k: attention(**{"D": 64, **k}),
    }
    return table[name](**kw)


def algorithmic_flops(p: Problem) -> int:
    """FLOPs of a contraction (``2MNK`` for matmul, ``4 B H S^2 D`` for
    attention); 0 for memory-bound kernels."""
    return int((p.oracle or {}).get("flops", 0))


def algorithmic_bytes(p: Problem) -> int:
    """Bytes a kernel must move at minimum: every input read once, every
    output written once (the roofline numerator for HBM-bound kernels)."""
    n = 0
    for _, shape, dt, _ in p.inputs:
        n += math.prod(shape) * (2 if dt == "bf16" else 4)
    n += 4 * len(p.consts)
    n += math.prod(p.out[1]) * 4 if p.out[1] else 4
    return n


def tma_scale(rows: int = 512, box_rows: int = 32, box_cols: int = 64, boxes: int = 2,
              block: int = 128, declare_mbar: bool = True) -> Problem:
    """``y = 2 x + 1`` over x f32[rows, boxes * box_cols], staged through shared
    memory with the TMA statements the reference defines but does not lower
    (TmaDescriptor, TmaLoad, MbarrierInit / ArriveExpectTx / Wait, SetMaxNReg):
    each CTA's thread 0 loads ``boxes`` boxes of box_rows x box_cols, one
    mbarrier slot each; every thread waits, then reads shared memory."""
    cols = boxes * box_cols
    p = Problem(f"tma_scale_{rows}x{cols}", "2 * x + 1", "k_tma_scale", "y")
    p.add_input("x", (rows, cols))
    p.out = ("y", (rows, cols), "f32")
    t0 = eq(V("a1_co"), Lit(0))
    body = [I.SetMaxNReg(64, "dec"),
            I.Smem("tile", (boxes, box_rows, box_cols), "float", 1024)]
    if declare_mbar:
        body.append(I.Smem("bar", (boxes,), "uint64_t", 8))
    body += [I.TmaDescriptor("xd", "x", (rows, cols), (box_rows, box_cols), "NONE", F32),
             I.Cond(t0, tuple(I.MbarrierInit("bar", 1, i) for i in range(boxes)), ()),
             I.Sync(0, None, False)]
    issue = []
    for i in range(boxes):
        issue += [I.MbarrierArriveExpectTx("bar", box_rows * box_cols * 4, i),
                  I.TmaLoad("tile", (Lit(i), Lit(0), Lit(0)), "xd",
                            (mul(V("a0"), Lit(box_rows)), Lit(i * box_cols)), "bar", i)]
    body.append(I.Cond(t0, tuple(issue), ()))
    for i in range(boxes):
        body.append(I.MbarrierWait("bar", 0, i))
        inner = strided(axis("c", box_cols), V("a1_co"), block, [
            load("v", "tile", Lit(i), V("r"), V("c")),
            I.Let("two", Lit(2.0), F32), I.Let("one", Lit(1.0), F32),
            assign("v2", "multiply", "v", "two"), assign("v3", "add", "v2", "one"),
            write("y", (add(mul(V("a0"), Lit(box_rows)), V("r")), add(Lit(i * box_cols), V("c"))),
                  ("v3",))])
        body.append(I.Loop(axis("r", box_rows), (inner,), False, False))
    p.body = tile([axis("a0", rows // box_rows), axis("a1_co", block)], body)
    p.grid, p.block = (rows // box_rows, 1, 1), (block, 1, 1)
    p.rtol, p.atol = 0, 0
    return p


def mbarrier_timeout(n: int = 1024, block: int = 128) -> Problem:
    """An mbarrier wait that no arrival completes: the bounded wait gives up
    after 2 s of %globaltimer, records status 8 in ``__emmy_status`` and the
    kernel finishes (``y = x``) -- the failure path, with no fault and no hang."""
    p = Problem(f"mbar_timeout_{n}", "x", "k_mbar_timeout", "y")
    p.add_input("x", (n,))
    p.out = ("y", (n,), "f32")
    p.body = tile([axis("a0", n)], [
        I.Smem("bar", (1,), "uint64_t", 8),
        I.Cond(eq(V("a0"), Lit(0)), (I.MbarrierInit("bar", 2, 0),), ()),
        I.Sync(0, None, False),
        I.Cond(eq(V("a0"), Lit(0)), (I.MbarrierWait("bar", 0, 0),), ()),
        load("v", "x", V("a0")), write("y", (V("a0"),), ("v",))])
    p.grid, p.block = (n // block, 1, 1), (block, 1, 1)
    p.rtol, p.atol = 0, 0
    return p


# --------------------------------------------------------------------------
# IR nodes the vocabulary defines but no reference IR uses (TASK.md rows
# marked *): small IRs written from the table's own descriptions
# --------------------------------------------------------------------------

def carried_prefix(rows: int = 64, cols: int = 96, every: int = 1, block: int = 64) -> Problem:
    """``Carry``/``Pre``: one thread per row steps through the columns with a
    carried cell ``c`` (seed 0): each step reads the previous state, and on
    steps where ``col % every == 0`` sets ``c = previous + x[row, col]``;
    ``y[row, col]`` is the state the step read -- the sum of the earlier
    columns that set it (other steps leave the cell as it was)."""
    p = Problem(f"carry_{rows}x{cols}_{every}", "exclusive prefix sum over every-th column",
                "k_carry", "y")
    p.add_input("x", (rows, cols))
    p.out = ("y", (rows, cols), "f32")
    step = [load("xv", "x", V("a0"), V("j")),
            I.Pre("prev", "c", ()),
            I.Cond(eq(I.BinaryExpr("%", V("j"), Lit(every)), Lit(0)),
                   (assign("nxt", "add", "prev", "xv"), I.Carry("c", "nxt", (), 0.0, F32)), ()),
            I.Pre("seen", "c", ()),
            write("y", (V("a0"), V("j")), ("seen",))]
    p.body = tile([axis("a0", rows)], [I.Loop(axis("j", cols), tuple(step), False, False)])
    p.grid, p.block = (-(-rows // block), 1, 1), (block, 1, 1)
    p.rtol, p.atol = 1e-5, 1e-5
    p.oracle = {"family": "carried_prefix", "args": {"x": "x"}, "output": "y", "every": every}
    return p


def select_branches(n: int = 4096, split: int = 1000, block: int = 256) -> Problem:
    """``Select``: y[i] = x[i] where i < split, else x[i] * x[i] -- the value
    of the branch whose coordinate predicate holds."""
    p = Problem(f"select_{n}", "where(i < split, x, x*x)", "k_select", "y")
    p.add_input("x", (n,))
    p.out = ("y", (n,), "f32")
    lt = I.BinaryExpr("<", V("a0"), Lit(split))
    ge = I.BinaryExpr(">=", V("a0"), Lit(split))
    p.body = tile([axis("a0", n)], [load("xv", "x", V("a0")), assign("sq", "multiply", "xv", "xv"),
                                    I.Select("v", (("xv", lt), ("sq", ge))),
                                    write("y", (V("a0"),), ("v",))])
    p.grid, p.block = (-(-n // block), 1, 1), (block, 1, 1)
    p.rtol, p.atol = 0, 0
    p.oracle = {"family": "select", "args": {"x": "x"}, "output": "y", "split": split}
    return p


def zero_prologue(words: int = 100_000, n: int = 4096, block: int = 128) -> Problem:
    """``ZeroPrologue``: the kernel zeroes the first ``words`` words of its
    output ``acc`` (another kernel's atomic accumulator in the vocabulary's
    use), every thread of the grid a strided share, and then adds x[i] into
    acc[i] atomically for its own cell."""
    p = Problem(f"zero_prologue_{words}", "acc[:words] = 0, then acc[:n] += x", "k_zero_pro",
                "acc")
    p.add_input("x", (n,))
    p.out = ("acc", (max(words, n),), "f32")
    p.body = tile([axis("a0", n)], [I.ZeroPrologue("acc", words), I.Sync(0, None, False),
                                    load("xv", "x", V("a0")),
                                    write("acc", (V("a0"),), ("xv",), atomic=True)])
    p.grid, p.block = (-(-n // block), 1, 1), (block, 1, 1)
    p.rtol, p.atol = 0, 0
    p.oracle = {"family": "zero_prologue", "args": {"x": "x"}, "output": "acc", "words": words}
    return p


# --------------------------------------------------------------------------
# the register-fragment tensor-core statements (mma.sync), written in the
# forms emmy_b200.fragments documents
# --------------------------------------------------------------------------

F16 = I.data_type("f16")


def _idiv(a, b):
    return I.BinaryExpr("/", a, Lit(b))


def _imod(a, b):
    return I.BinaryExpr("%", a, Lit(b))


def _and(a, b):
    return I.BinaryExpr("&&", a, b)


def _xor(a, b):
    return I.BinaryExpr("^", a, b)


def mma_matmul(M: int = 200, N: int = 136, K: int = 80, dtype: str = "bf16",
               b_kn: bool = True, stage: bool = True, promote: bool = False,
               epilogue: bool = False, out_dtype: str = "f32", split_k: int = 1,
               swizzle: bool = False) -> Problem:
    """C = A . B through register fragments: CTAs of 128 threads own 64 x 64
    tiles of C, each warp a 32 x 32 quarter as 2 x 4 mma.sync atoms.

    ``dtype`` bf16 / f16 (m16n8k16) or tf32 (f32 inputs, m16n8k8); ``b_kn``:
    B is given [K, N] (fragments loaded transposed) or as Bt [N, K];
    ``stage``: 64 x 32 slabs of A and B staged in shared memory by the
    CTA's threads (ldmatrix for 16-bit operands), else fragments loaded
    straight from global memory with row / column and K guards;
    ``promote``: f16 products accumulated in f16 fragments, added into the
    f32 accumulators after every slab; ``epilogue``: C = relu(A.B + bias[col])
    through the store's Lambda; ``out_dtype`` f32 or bf16; ``split_k`` > 1:
    that many CTAs per tile, each over a K range, adding atomically into a
    zeroed C.  ``swizzle`` (16-bit, staged): 64-wide slabs without padding,
    written with their 16-byte chunks XOR-swizzled by row (chunk c of row r at
    c ^ (r % 8)) and read back by ldmatrix through the ``"B128"`` swizzle."""
    wide = dtype in ("bf16", "f16")
    in_dt = {"bf16": BF16, "f16": F16, "tf32": F32}[dtype]
    in_name = {"bf16": "bf16", "f16": "f16", "tf32": "f32"}[dtype]
    shape = "m16n8k16" if wide else "m16n8k8"
    KK = 16 if wide else 8
    BK, MI, NJ = (64 if swizzle else 32), 2, 4
    pad = 0 if swizzle else (8 if wide else 4)
    swz = "B128" if swizzle else None
    smem_ty = {"bf16": "bfloat16", "f16": "half", "tf32": "float"}[dtype]
    kper = -(-K // split_k)
    nk = -(-kper // BK)
    p = Problem(f"mma_matmul_{dtype}_{M}x{N}x{K}", "a @ b", "k_mma_matmul", "c")
    p.add_input("a", (M, K), in_name)
    p.add_input("b", (K, N) if b_kn else (N, K), in_name)
    if epilogue:
        p.add_input("bias", (N,))
    p.out = ("c", (M, N), out_dtype)
    t = V("t")
    body = [I.Let("w", _idiv(t, 32), I.data_type("i32")),
            I.Let("wm", _idiv(V("w"), 2), I.data_type("i32")),
            I.Let("wn", _imod(V("w"), 2), I.data_type("i32")),
            I.Let("rowbase", add(mul(V("bm"), Lit(64)), mul(V("wm"), Lit(32))), I.data_type("i32")),
            I.Let("colbase", add(mul(V("bn"), Lit(64)), mul(V("wn"), Lit(32))), I.data_type("i32")),
            I.Let("kend", I.BinaryExpr("min", add(mul(V("ks"), Lit(kper)), Lit(kper)), Lit(K)),
                  I.data_type("i32")),
            I.Let("zero", Lit(0.0), F32),
            I.RegFragment("acc", "c", shape, F32, MI * NJ, 4),
            I.RegFragment("fa", "a", shape, dtype, MI, 4 if (wide or KK == 8) else 2),
            I.RegFragment("fb", "b", shape, dtype, NJ, 2)]
    if promote:
        body.append(I.RegFragment("acch", "c", shape, F16, MI * NJ, 2))
    acc = "acch" if promote else "acc"
    if stage:
        body += [I.Smem("As", (64, BK + pad), smem_ty, 128),
                 I.Smem("Bs", (BK, 64 + pad) if b_kn else (64, BK + pad), smem_ty, 128)]
    slab = [I.Let("k0", add(mul(V("ks"), Lit(kper)), mul(V("kt"), Lit(BK))), I.data_type("i32"))]
    if stage:
        def stage_copy(dst, src, rows, cols, src_r, src_c, rbound, cbound):
            r, c = _idiv(V("e"), cols), _imod(V("e"), cols)
            ok = _and(I.BinaryExpr("<", src_r(r), rbound), I.BinaryExpr("<", src_c(c), cbound))
            dc = _xor(c, mul(_imod(r, 8), Lit(8))) if swizzle else c
            return strided(axis("e", rows * cols), t, 128, [
                I.Cond(ok, (load("v", src, src_r(r), src_c(c), dtype=in_dt),
                            write(dst, (r, dc), ("v",))),
                       (write(dst, (r, dc), ("zero",)),))])
        slab.append(stage_copy("As", "a", 64, BK, lambda r: add(mul(V("bm"), Lit(64)), r),
                               lambda c: add(V("k0"), c), Lit(M), V("kend")))
        if b_kn:
            slab.append(stage_copy("Bs", "b", BK, 64, lambda r: add(V("k0"), r),
                                   lambda c: add(mul(V("bn"), Lit(64)), c), V("kend"), Lit(N)))
        else:
            slab.append(stage_copy("Bs", "b", 64, BK, lambda r: add(mul(V("bn"), Lit(64)), r),
                                   lambda c: add(V("k0"), c), Lit(N), V("kend")))
        slab.append(I.Sync(0, None, False))
    for kk in range(BK // KK):
        for i in range(MI):
            if stage:
                slab.append(I.LdmatrixLoad(f"fa[{i}]", "As", (add(mul(V("wm"), Lit(32)), Lit(16 * i)),
                                                           Lit(kk * KK)), "a", BK + pad, swz))
            else:
                slab.append(I.LdmatrixLoad(f"fa[{i}]", "a", (add(V("rowbase"), Lit(16 * i)),
                                                          add(V("k0"), Lit(kk * KK))), "a",
                                           gmem_guard=(Lit(M), None), k_zero=V("kend")))
        for j in range(NJ):
            if stage:
                n_off = add(mul(V("wn"), Lit(32)), Lit(8 * j))
                idx = (Lit(kk * KK), n_off) if b_kn else (n_off, Lit(kk * KK))
                slab.append(I.LdmatrixLoad(f"fb[{j}]", "Bs", idx, "b",
                                           (64 + pad) if b_kn else (BK + pad), swz, b_trans=b_kn))
            else:
                n_abs = add(V("colbase"), Lit(8 * j))
                k_abs = add(V("k0"), Lit(kk * KK))
                idx = (k_abs, n_abs) if b_kn else (n_abs, k_abs)
                guard = (None, Lit(N)) if b_kn else (Lit(N), None)
                slab.append(I.LdmatrixLoad(f"fb[{j}]", "b", idx, "b", gmem_guard=guard,
                                           k_zero=V("kend"), b_trans=b_kn))
        for i in range(MI):
            for j in range(NJ):
                slab.append(I.MmaSyncPtx(f"{acc}[{i * NJ + j}]", f"fa[{i}]", f"fb[{j}]", shape,
                                         dtype, "f16" if promote else F32))
    if stage:
        slab.append(I.Sync(0, None, False))
    if promote:
        slab += [I.FragmentPromote(f"acc[{c}]", f"acch[{c}]") for c in range(MI * NJ)]
    body.append(I.Loop(axis("kt", nk), tuple(slab), False, False))
    lam = None
    if epilogue:
        lam = I.Lambda(("v",), (load("bv", "bias", V("col")), I.Let("z0", Lit(0.0), F32),
                                assign("s", "add", "v", "bv"), assign("o", "maximum", "s", "z0")),
                       ("o",))
    for i in range(MI):
        for j in range(NJ):
            body.append(I.RegStore("c", (add(V("rowbase"), Lit(16 * i)), add(V("colbase"), Lit(8 * j))),
                                   f"acc[{i * NJ + j}]", shape, None, lam, (), Lit(M), Lit(N),
                                   split_k > 1))
    gm, gn = -(-M // 64), -(-N // 64)
    p.body = I.Tile((axis("ks", split_k), axis("bm", gm), axis("bn", gn), axis("t", 128)),
                    tuple(body), 128)
    p.grid, p.block = (split_k * gm * gn, 1, 1), (128, 1, 1)
    if split_k > 1:
        p.zero = ["c"]
    p.rtol = {"bf16": 1e-3, "f16": 2e-2 if promote else 1e-3, "tf32": 5e-3}[dtype]
    if out_dtype == "bf16":
        p.rtol = max(p.rtol, 1e-2)
    p.atol = None
    p.oracle = {"family": "mma_matmul", "args": {"a": "a", "b": "b", "bias": "bias"},
                "output": "c", "b_kn": b_kn, "epilogue": epilogue, "tf32": dtype == "tf32",
                "bf16": {"a": dtype == "bf16", "b": dtype == "bf16"}, "out_bf16": out_dtype == "bf16"}
    return p


def mma_attention(Sq: int = 128, Sk: int = 64, d: int = 32, causal: bool = False,
                  bias: bool = False, scale: float | None = None) -> Problem:
    """O = softmax(Q K^T * scale (+ bias) (masked: key <= query)) V for bf16
    Q [Sq, d], K, V [Sk, d]: each warp owns 16 query rows and all Sk keys
    in registers -- S by mma.sync from Q fragments read from global memory and
    K fragments from shared memory, the row max and row sum by
    FragmentRowReduce, P = 2^(S c - max) by FragmentApply (mask and bias
    arguments too; the bias row clamped to the last query, so the rows of a
    ragged last block past Sq read in bounds), P repacked as bf16 A fragments
    (FragmentRepack), O = P V, O / l by a row argument, stored by RegStore."""
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    c = scale * 1.4426950408889634
    nS, nD, nK16 = Sk // 8, d // 8, Sk // 16
    p = Problem(f"mma_attention_{Sq}x{Sk}x{d}", "softmax(q k^T s) v", "k_mma_attention", "o")
    p.add_input("q", (Sq, d), "bf16")
    p.add_input("k", (Sk, d), "bf16")
    p.add_input("v", (Sk, d), "bf16")
    if bias:
        p.add_input("bias", (Sq, Sk))
    p.out = ("o", (Sq, d), "f32")
    t = V("t")
    i32 = I.data_type("i32")
    body = [I.Let("w", _idiv(t, 32), i32),
            I.Let("qrow", add(mul(V("qb"), Lit(64)), mul(V("w"), Lit(16))), i32),
            I.Smem("Ks", (Sk, d + 8), "bfloat16", 128), I.Smem("Vs", (Sk, d + 8), "bfloat16", 128)]
    for sm, src in (("Ks", "k"), ("Vs", "v")):
        r, cc = _idiv(V("e"), d), _imod(V("e"), d)
        body.append(strided(axis("e", Sk * d), t, 128, [load("x", src, r, cc, dtype=BF16),
                                                          write(sm, (r, cc), ("x",))]))
    body += [I.Sync(0, None, False),
             I.RegFragment("fq", "a", "m16n8k16", BF16, d // 16, 4),
             I.RegFragment("fk", "b", "m16n8k16", BF16, 1, 2),
             I.RegFragment("s", "c", "m16n8k16", F32, nS, 4),
             I.RegFragment("fp", "a", "m16n8k16", BF16, nK16, 4),
             I.RegFragment("fv", "b", "m16n8k16", BF16, 1, 2),
             I.RegFragment("o", "c", "m16n8k16", F32, nD, 4),
             I.Let("c", Lit(c), F32), I.Let("ninf", Lit(float("-inf")), F32),
             I.Let("log2e", Lit(1.4426950408889634), F32)]
    for kk in range(d // 16):
        body.append(I.LdmatrixLoad(f"fq[{kk}]", "q", (V("qrow"), Lit(16 * kk)), "a",
                                   gmem_guard=(Lit(Sq), None)))
    for j in range(nS):
        for kk in range(d // 16):
            body += [I.LdmatrixLoad("fk", "Ks", (Lit(8 * j), Lit(16 * kk)), "b", d + 8, b_trans=False),
                     I.MmaSyncPtx(f"s[{j}]", f"fq[{kk}]", "fk", "m16n8k16", BF16, F32)]
    for j in range(nS):
        body.append(I.FragmentApply(f"s[{j}]", "multiply", (f"s[{j}]", "c"), ("frag", "scalar")))
        if bias:
            # s + bias * log2(e): the scores are in base-2 units from here on
            brow = I.BinaryExpr("min", V("row"), Lit(Sq - 1))
            body.append(I.FragmentApply(f"s[{j}]", "fma",
                                        (("bias", (brow, V("col"))), "log2e", f"s[{j}]"),
                                        ("bias", "scalar", "frag"), True, None, None,
                                        V("qrow"), Lit(8 * j)))
        if causal:
            body.append(I.FragmentApply(f"s[{j}]", "where",
                                        (I.BinaryExpr("<=", V("col"), V("row")), f"s[{j}]", "ninf"),
                                        ("mask", "frag", "scalar"), True, None, None,
                                        V("qrow"), Lit(8 * j)))
    body.append(I.FragmentRowReduce("mt", "mb", tuple(f"s[{j}]" for j in range(nS)), "max"))
    for j in range(nS):
        body.append(I.FragmentApply(f"s[{j}]", "subtract", (f"s[{j}]", ("mt", "mb")),
                                    ("frag", "row"), True, None, "exp2"))
    body.append(I.FragmentRowReduce("lt", "lb", tuple(f"s[{j}]" for j in range(nS)), "add"))
    for i in range(nK16):
        body.append(I.FragmentRepack(f"fp[{i}]", tuple(f"s[{j}]" for j in range(nS)), BF16, None, i))
    for i in range(nK16):
        for j in range(nD):
            body += [I.LdmatrixLoad("fv", "Vs", (Lit(16 * i), Lit(8 * j)), "b", d + 8, b_trans=True),
                     I.MmaSyncPtx(f"o[{j}]", f"fp[{i}]", "fv", "m16n8k16", BF16, F32)]
    for j in range(nD):
        body += [I.FragmentApply(f"o[{j}]", "divide", (f"o[{j}]", ("lt", "lb")), ("frag", "row")),
                 I.RegStore("o", (V("qrow"), Lit(8 * j)), f"o[{j}]", "m16n8k16", m_guard=Lit(Sq))]
    gq = -(-Sq // 64)
    p.body = I.Tile((axis("qb", gq), axis("t", 128)), tuple(body), 128)
    p.grid, p.block = (gq, 1, 1), (128, 1, 1)
    p.rtol, p.atol = 2e-2, None
    p.oracle = {"family": "mma_attention", "args": {"q": "q", "k": "k", "v": "v", "bias": "bias"},
                "output": "o", "scale": scale, "causal": causal, "bias_on": bias,
                "bf16": {"q": True, "k": True, "v": True}}
    return p


def wgmma_matmul(M: int = 200, N: int = 136, K: int = 200, BN: int = 64, layout: str = "sw128",
                 warpgroups: int = 1, pipelined: bool = False, dtype: str = "bf16",
                 a_regs: bool = False) -> Problem:
    """C = A . B through the warpgroup statements (WgmmaDescriptor, WgmmaFence,
    WgmmaMma m64nBNk16, WgmmaCommit, WgmmaWait): each warpgroup owns 64 rows
    of a CTA tile of 64 * ``warpgroups`` x BN, the CTA's threads stage 64-wide
    K slabs of A and B into shared memory in the canonical layout the
    descriptors name, and each warp stores its 16 rows of the accumulator with
    RegStore.  ``layout``: ``sw128`` (both operands K-major, 128-byte
    swizzle: element (r, k) of a 64-wide slab at r*64 + ((k/8 ^ r%8)*8) +
    k%8), ``sw128_mn`` (B MN-major, 128-byte swizzle, 64-column blocks of
    64 k-rows, LBO between blocks) or ``none`` (K-major without swizzle:
    8x8 core matrices, LBO 128 B between core matrices along K, SBO 1024 B
    between 8-row groups).  ``pipelined``: two slab buffers, a commit per
    slab and ``WgmmaWait(1)`` before a buffer is refilled.  ``a_regs``: the A
    operand in registers -- each warp loads its 16 rows of every 16-wide K
    step as an A fragment straight from global memory (guarded) and passes
    it as ``a_frag``."""
    dt = {"bf16": BF16, "f16": F16, "tf32": F32}[dtype]
    smem_ty = {"bf16": "bfloat16", "f16": "half", "tf32": "float"}[dtype]
    es = 4 if dtype == "tf32" else 2           # bytes an element
    ce = 16 // es                              # elements a 16-byte chunk
    BK = 128 // es                             # a 128-byte row of K a slab
    KS = 8 if dtype == "tf32" else 16          # K of one product
    if dtype == "tf32" and (layout == "sw128_mn" or a_regs):
        raise ValueError("tf32 operands: K-major shared memory only")
    BM = 64 * warpgroups
    T = 128 * warpgroups
    nbuf = 2 if pipelined else 1
    nk = -(-K // BK)
    p = Problem(f"wgmma_matmul_{layout}_{M}x{N}x{K}", "a @ b", "k_wgmma_matmul", "c")
    p.add_input("a", (M, K), "f32" if dtype == "tf32" else dtype)
    p.add_input("b", (K, N), "f32" if dtype == "tf32" else dtype)
    p.out = ("c", (M, N), "f32")
    t = V("t")
    i32 = I.data_type("i32")
    a_sz, b_sz = BM * BK, BN * BK

    def pos_kmajor(r, kk):
        if layout == "none":
            return add(add(mul(_idiv(r, 8), Lit(1024 // es)), mul(_idiv(kk, ce), Lit(128 // es))),
                       add(mul(_imod(r, 8), Lit(ce)), _imod(kk, ce)))
        return add(mul(r, Lit(BK)), add(mul(_xor(_idiv(kk, ce), _imod(r, 8)), Lit(ce)),
                                        _imod(kk, ce)))

    def pos_mn(kk, n):
        return add(add(mul(_idiv(n, 64), Lit(64 * BK)), mul(kk, Lit(64))),
                   add(mul(_xor(_idiv(_imod(n, 64), 8), _imod(kk, 8)), Lit(8)), _imod(n, 8)))

    body = [I.Let("w", _idiv(t, 32), i32), I.Let("wg", _idiv(t, 128), i32),
            I.Let("zero", Lit(0.0), F32),
            I.Smem("As", (nbuf * a_sz,), smem_ty, 1024), I.Smem("Bs", (nbuf * b_sz,), smem_ty, 1024),
            I.RegFragment("acc", "c", "m16n8k16", F32, BN // 8, 4)]
    if a_regs:
        body.append(I.RegFragment("fa", "a", "m16n8k16", dt, 1, 4))
    slab = [I.Let("k0", mul(V("kt"), Lit(BK)), i32),
            I.Let("buf", _imod(V("kt"), nbuf) if nbuf > 1 else Lit(0), i32)]
    if pipelined:
        slab.append(I.WgmmaWait(1))
    r, kk = _idiv(V("e"), BK), _imod(V("e"), BK)
    arow = add(mul(V("bm"), Lit(BM)), r)
    a_stage = strided(axis("e", BM * BK), t, T, [
        I.Cond(_and(I.BinaryExpr("<", arow, Lit(M)), I.BinaryExpr("<", add(V("k0"), kk), Lit(K))),
               (load("v", "a", arow, add(V("k0"), kk), dtype=dt),
                write("As", (add(mul(V("buf"), Lit(a_sz)), pos_kmajor(r, kk)),), ("v",))),
               (write("As", (add(mul(V("buf"), Lit(a_sz)), pos_kmajor(r, kk)),), ("zero",)),))])
    if not a_regs:
        slab.append(a_stage)
    kr, n = _idiv(V("e"), BN), _imod(V("e"), BN)
    ncol = add(mul(V("bn"), Lit(BN)), n)
    bpos = pos_mn(kr, n) if layout == "sw128_mn" else pos_kmajor(n, kr)
    slab.append(strided(axis("e", BK * BN), t, T, [
        I.Cond(_and(I.BinaryExpr("<", add(V("k0"), kr), Lit(K)), I.BinaryExpr("<", ncol, Lit(N))),
               (load("v", "b", add(V("k0"), kr), ncol, dtype=dt),
                write("Bs", (add(mul(V("buf"), Lit(b_sz)), bpos),), ("v",))),
               (write("Bs", (add(mul(V("buf"), Lit(b_sz)), bpos),), ("zero",)),))]))
    slab += [I.Sync(0, None, False), I.WgmmaFence()]
    swz = "NONE" if layout == "none" else "128B"
    a_lbo, a_sbo = (128, 1024) if layout == "none" else (16, 1024)
    b_lbo, b_sbo = ((64 * BK * 2, 1024) if layout == "sw128_mn" else (a_lbo, a_sbo))
    for s in range(BK // KS):
        a_step = (KS // ce) * (128 // es) * s if layout == "none" else KS * s
        b_step = 16 * 64 * s if layout == "sw128_mn" else a_step
        a_idx = add(add(mul(V("buf"), Lit(a_sz)), mul(V("wg"), Lit(64 * BK))), Lit(a_step))
        b_idx = add(mul(V("buf"), Lit(b_sz)), Lit(b_step))
        first = I.BinaryExpr("||", I.BinaryExpr(">", V("kt"), Lit(0)), I.BinaryExpr(">", Lit(s), Lit(0)))
        scale = first if s == 0 else Lit(1)
        if a_regs:
            wrow = add(add(mul(V("bm"), Lit(BM)), mul(V("wg"), Lit(64))), mul(_imod(V("w"), 4), Lit(16)))
            slab += [I.LdmatrixLoad("fa", "a", (wrow, add(V("k0"), Lit(16 * s))), "a",
                                    gmem_guard=(Lit(M), None), k_zero=Lit(K)),
                     I.WgmmaDescriptor("db", "Bs", (b_idx,), swz, b_lbo, b_sbo),
                     I.WgmmaMma("acc", "db", f"m64n{BN}k{KS}", dt, None, "fa", scale, 0,
                                int(layout == "sw128_mn"))]
            continue
        slab += [I.WgmmaDescriptor("da", "As", (a_idx,), swz, a_lbo, a_sbo),
                 I.WgmmaDescriptor("db", "Bs", (b_idx,), swz, b_lbo, b_sbo),
                 I.WgmmaMma("acc", "db", f"m64n{BN}k{KS}",
                            I.data_type("tf32") if dtype == "tf32" else dt, "da", None,
                            scale, 0, int(layout == "sw128_mn"))]
    slab.append(I.WgmmaCommit())
    if not pipelined:
        slab.append(I.WgmmaWait(0))
    body.append(I.Loop(axis("kt", nk), tuple(slab), False, False))
    body.append(I.WgmmaWait(0))
    row0 = add(add(mul(V("bm"), Lit(BM)), mul(V("wg"), Lit(64))), mul(_imod(V("w"), 4), Lit(16)))
    for j in range(BN // 8):
        body.append(I.RegStore("c", (row0, add(mul(V("bn"), Lit(BN)), Lit(8 * j))), f"acc[{j}]",
                               m_guard=Lit(M), n_guard=Lit(N)))
    gm, gn = -(-M // BM), -(-N // BN)
    p.body = I.Tile((axis("bm", gm), axis("bn", gn), axis("t", T)), tuple(body), T)
    p.grid, p.block = (gm * gn, 1, 1), (T, 1, 1)
    p.rtol, p.atol = (5e-3 if dtype == "tf32" else 1e-3), None
    p.oracle = {"family": "mma_matmul", "args": {"a": "a", "b": "b", "bias": "bias"},
                "output": "c", "b_kn": True, "epilogue": False,
                "tf32": "trunc" if dtype == "tf32" else False,
                "bf16": {"a": dtype == "bf16", "b": dtype == "bf16"}, "out_bf16": False}
    return p

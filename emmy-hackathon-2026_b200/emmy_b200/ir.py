"""Kernel IR data model and a safe reader for Emmy's serialised IR graphs.

Emmy (emmy-ml 0.3.11) stores each KernelOp body as a list of Python ``repr``
strings of its statement dataclasses (see a problem's ``*.ir.json``,
``op_fields.body[0]``).  The reference loads them with
``emmy.compiler.graph.Graph.from_dict`` (reference ``compile.py:59-60,2641``).
emmy-ml is not installable offline, so this module restates that schema:

* every IR class named in the reference task's Kernel IR tables
  (reference ``TASK.md:64-188``) is a frozen dataclass with the same field
  names and order, so ``type(node).__name__`` and attribute access match the
  emmy objects the reference compiler walks;
* the ``repr`` strings are parsed with :mod:`ast` and rebuilt node by node --
  never ``eval`` -- so an IR file cannot run code.

When emmy-ml *is* importable, :func:`load_graph` prefers it (the north-star
contract); otherwise it falls back to this reader.  Both give objects with
the same attribute surface.
"""
from __future__ import annotations

import ast
import dataclasses
import json
from typing import Any

# ---------------------------------------------------------------------------
# node classes
# ---------------------------------------------------------------------------

_EXPR_MODULE = "emmy.compiler.ir.expr"
_STMT_MODULE = "emmy.compiler.ir.stmt"
_TYPE_MODULE = "emmy.compiler.ir.types"
_FRAG_MODULE = "emmy.compiler.ir.fragment"

# name -> (module, fields).  Field order follows the keyword order Emmy's
# dataclass reprs print, which is the declaration order.
_SCHEMA: dict[str, tuple[str, tuple[str, ...]]] = {
    # expressions (TASK.md "Expressions")
    "Var": (_EXPR_MODULE, ("name",)),
    "Literal": (_EXPR_MODULE, ("value", "dtype")),
    "BinaryExpr": (_EXPR_MODULE, ("op", "left", "right")),
    "TernaryExpr": (_EXPR_MODULE, ("cond", "if_true", "if_false")),
    "CastExpr": (_EXPR_MODULE, ("dtype", "expr")),
    "FlatIndex": (_EXPR_MODULE, ("buffer", "index")),
    "Builtin": (_EXPR_MODULE, ("name",)),
    "FuncCallExpr": (_EXPR_MODULE, ("name", "args")),
    # types and axes
    "DataType": (_TYPE_MODULE, ("name", "np", "nbytes")),
    "Dim": (_TYPE_MODULE, ("value",)),
    "Axis": (_TYPE_MODULE, ("name", "extent", "window")),
    "Window": (_TYPE_MODULE, ("parent", "base", "bound", "partition")),
    "ElementwiseImpl": (_TYPE_MODULE, ("name",)),
    # statements (TASK.md "Scalar compute", "Launch", "Transport", "Combine")
    "Tile": (_STMT_MODULE, ("axes", "body", "block_threads", "aux_threads",
                            "raster_axes", "raster_group", "raster_orient")),
    "StridedLoop": (_STMT_MODULE, ("axis", "start", "step", "body", "unroll", "end", "seed")),
    "Loop": (_STMT_MODULE, ("axis", "body", "unroll", "seed")),
    "Load": (_STMT_MODULE, ("names", "input", "index", "dtype")),
    "Assign": (_STMT_MODULE, ("name", "op", "args", "dtype")),
    "Let": (_STMT_MODULE, ("name", "value", "dtype")),
    "Accum": (_STMT_MODULE, ("name", "value", "op", "dtype", "axes", "base")),
    "Init": (_STMT_MODULE, ("name", "identity", "dtype")),
    "Write": (_STMT_MODULE, ("output", "index", "values", "value_dtype", "atomic", "swizzle")),
    "Cond": (_STMT_MODULE, ("cond", "body", "else_body")),
    "Smem": (_STMT_MODULE, ("name", "extents", "dtype", "align")),
    "Sync": (_STMT_MODULE, ("barrier_id", "count", "warp")),
    "WarpShuffle": (_STMT_MODULE, ("state", "state_b", "combine_states", "length", "dtype")),
    "TreeHalve": (_STMT_MODULE, ("bufs", "state", "state_b", "combine_states", "length",
                                 "tid_var", "dtype", "barrier_id", "barrier_count", "inner")),
    "CpAsyncCopy": (_STMT_MODULE, ("smem", "smem_index", "src", "src_index", "nbytes",
                                   "swizzle", "lane_index", "lane_rows")),
    "CpAsyncCommit": (_STMT_MODULE, ()),
    "CpAsyncWait": (_STMT_MODULE, ("group",)),
    # defined by the IR vocabulary but used by no problem (TASK.md rows marked *)
    "Pre": (_STMT_MODULE, ("name", "carrier", "index")),
    "Carry": (_STMT_MODULE, ("name", "value", "index", "seed", "dtype")),
    "Select": (_STMT_MODULE, ("name", "branches")),
    "ZeroPrologue": (_STMT_MODULE, ("dst", "words")),
    "TmaDescriptor": (_STMT_MODULE, ("name", "src_buf", "src_shape", "box_extents", "swizzle", "dtype")),
    "TmaLoad": (_STMT_MODULE, ("smem", "smem_index", "desc", "coords", "mbar", "mbar_slot")),
    "MbarrierInit": (_STMT_MODULE, ("mbar", "count", "slot")),
    "MbarrierArriveExpectTx": (_STMT_MODULE, ("mbar", "bytes_", "slot")),
    "MbarrierArrive": (_STMT_MODULE, ("mbar", "slot")),
    "MbarrierWait": (_STMT_MODULE, ("mbar", "phase", "slot")),
    "SetMaxNReg": (_STMT_MODULE, ("count", "direction")),
    # tensor core through register fragments (mma.sync), TASK.md "Tensor core:
    # register fragments"; Lambda and FragLayout are the helper records those
    # statements carry
    "RegFragment": (_STMT_MODULE, ("name", "role", "shape", "dtype", "count", "nregs")),
    "LdmatrixLoad": (_STMT_MODULE, ("frag", "src_buffer", "src_index", "role", "ldm", "swizzle",
                                    "staged", "gmem_guard", "k_zero", "b_trans", "pair_frag",
                                    "byte_slab", "scale_buffer", "scale_index", "scale_ldm",
                                    "fragment_layout", "fragment_index")),
    "BlockScaleLoad": (_STMT_MODULE, ("frag", "src_buffer", "src_index", "role", "ldm")),
    "MmaSyncPtx": (_STMT_MODULE, ("c_frag", "a_frag", "b_frag", "shape", "ab_dtype", "c_dtype",
                                  "b_row_major", "sfa_frag", "sfb_frag")),
    "FragmentPromote": (_STMT_MODULE, ("dst", "src")),
    "FragmentApply": (_STMT_MODULE, ("out", "op", "args", "kinds", "in_place", "layout", "post",
                                     "row_base", "col_base")),
    "FragmentRowReduce": (_STMT_MODULE, ("top", "bot", "frags", "op", "layout", "dtype")),
    "FragmentRepack": (_STMT_MODULE, ("frag", "srcs", "ab_dtype", "fragment_layout", "part")),
    "RegStore": (_STMT_MODULE, ("dst_buffer", "dst_index", "frag", "shape", "ldm", "epilogue",
                                "extra_frags", "m_guard", "n_guard", "atomic", "fragment_layout",
                                "volta_interleaved", "fragment_index", "swizzle", "row_dim",
                                "col_dim")),
    "Lambda": (_FRAG_MODULE, ("params", "body", "results")),
    "FragLayout": (_FRAG_MODULE, ("n_elems", "elem_row", "reduce_xors", "lane_decl", "lane_names",
                                  "row_off", "col_off")),
    # tensor core through warpgroups (wgmma), TASK.md "Tensor core: warp groups"
    "WgmmaDescriptor": (_STMT_MODULE, ("name", "smem", "smem_index", "swizzle", "lbo_bytes",
                                       "sbo_bytes")),
    "WgmmaMma": (_STMT_MODULE, ("c_frags", "b_desc", "shape", "ab_dtype", "a_desc", "a_frag",
                                "scale_d", "trans_a", "trans_b")),
    "WgmmaFence": (_STMT_MODULE, ()),
    "WgmmaCommit": (_STMT_MODULE, ()),
    "WgmmaWait": (_STMT_MODULE, ("group",)),
}

_DEFAULTS: dict[str, dict[str, Any]] = {
    "Axis": {"window": None},
    "Literal": {"dtype": "int"},
    "Tile": {"block_threads": None, "aux_threads": 0, "raster_axes": None,
             "raster_group": None, "raster_orient": "m"},
    "StridedLoop": {"unroll": False, "end": None, "seed": False},
    "Loop": {"unroll": False, "seed": False},
    "Accum": {"axes": (), "base": None},
    "Write": {"atomic": False, "swizzle": "NONE"},
    "Cond": {"else_body": ()},
    "Smem": {"align": 0},
    "Sync": {"barrier_id": 0, "count": None, "warp": False},
    "TreeHalve": {"barrier_id": 0, "barrier_count": None, "inner": None},
    "CpAsyncCopy": {"swizzle": None, "lane_index": None, "lane_rows": None},
    "CpAsyncWait": {"group": 0},
    "Window": {"base": None, "bound": None, "partition": False},
    "RegFragment": {"count": 1, "nregs": None},
    "LdmatrixLoad": {"role": None, "ldm": None, "swizzle": None, "staged": False,
                     "gmem_guard": None, "k_zero": None, "b_trans": False, "pair_frag": None,
                     "byte_slab": None, "scale_buffer": None, "scale_index": None,
                     "scale_ldm": None, "fragment_layout": None, "fragment_index": None},
    "BlockScaleLoad": {"ldm": None},
    "MmaSyncPtx": {"shape": None, "ab_dtype": None, "c_dtype": None, "b_row_major": False,
                   "sfa_frag": None, "sfb_frag": None},
    "FragmentApply": {"kinds": (), "in_place": True, "layout": None, "post": None,
                      "row_base": None, "col_base": None},
    "FragmentRowReduce": {"layout": None, "dtype": None},
    "FragmentRepack": {"ab_dtype": None, "fragment_layout": None, "part": 0},
    "RegStore": {"shape": None, "ldm": None, "epilogue": None, "extra_frags": (), "m_guard": None,
                 "n_guard": None, "atomic": False, "fragment_layout": None,
                 "volta_interleaved": False, "fragment_index": None, "swizzle": None,
                 "row_dim": None, "col_dim": None},
    "FragLayout": {"reduce_xors": (1, 2), "lane_decl": (), "lane_names": ()},
    "WgmmaDescriptor": {"swizzle": "NONE", "lbo_bytes": 0, "sbo_bytes": 0},
    "WgmmaMma": {"ab_dtype": None, "a_desc": None, "a_frag": None, "scale_d": 1, "trans_a": 0,
                 "trans_b": 0},
    "WgmmaWait": {"group": 0},
}


def _free_vars(self) -> set[str]:
    """Names an expression reads (the attribute the reference's use census
    calls on expression nodes, reference ``compile.py:134-135``)."""
    out: set[str] = set()

    def walk(e):
        k = type(e).__name__
        if k == "Var":
            out.add(e.name)
        elif k == "BinaryExpr":
            walk(e.left)
            walk(e.right)
        elif k == "TernaryExpr":
            walk(e.cond)
            walk(e.if_true)
            walk(e.if_false)
        elif k == "CastExpr":
            walk(e.expr)
        elif k == "FlatIndex":
            for i in e.index:
                walk(i)
        elif k == "FuncCallExpr":
            for a in e.args:
                walk(a)

    walk(self)
    return out


def _make_class(name: str, module: str, fields: tuple[str, ...]):
    defaults = _DEFAULTS.get(name, {})
    spec = []
    seen_default = False
    for f in fields:
        if f in defaults:
            spec.append((f, Any, dataclasses.field(default=defaults[f])))
            seen_default = True
        elif seen_default:
            spec.append((f, Any, dataclasses.field(default=None)))
        else:
            spec.append((f, Any))
    ns = {}
    if module == _EXPR_MODULE:
        ns["free_vars"] = _free_vars
    cls = dataclasses.make_dataclass(name, spec, frozen=True, namespace=ns)
    cls.__module__ = module
    cls.__qualname__ = name
    return cls


class _NodeClasses(dict):
    """name -> IR class, each made the first time it is asked for (an IR
    names only a few of the vocabulary's classes; making all of them costs
    a one-kernel ``compile.py`` run tens of milliseconds).  ``in`` and
    iteration see the whole vocabulary."""

    def __missing__(self, name):
        if name not in _SCHEMA:
            raise KeyError(name)
        m, f = _SCHEMA[name]
        cls = self[name] = _make_class(name, m, f)
        return cls

    def get(self, name, default=None):
        return self[name] if name in _SCHEMA else default

    def __contains__(self, name):
        return name in _SCHEMA

    def __iter__(self):
        return iter(_SCHEMA)

    def keys(self):
        return list(_SCHEMA)

    def items(self):
        return [(n, self[n]) for n in _SCHEMA]

    def values(self):
        return [self[n] for n in _SCHEMA]

    def __len__(self):
        return len(_SCHEMA)


NODE_CLASSES: dict[str, type] = _NodeClasses()


def __getattr__(name):
    """``ir.Tile``, ``from .ir import Var`` and the like: the class, made on
    first use."""
    if name in _SCHEMA:
        return NODE_CLASSES[name]
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")

STMT_KINDS = frozenset(n for n, (m, _) in _SCHEMA.items() if m == _STMT_MODULE)
EXPR_KINDS = frozenset(n for n, (m, _) in _SCHEMA.items() if m == _EXPR_MODULE)


class NpDtype(str):
    """Stand-in for the ``numpy.dtype('float32')`` carried inside ``DataType``;
    compares and hashes as its name."""


# ---------------------------------------------------------------------------
# safe repr parser
# ---------------------------------------------------------------------------


class IRParseError(ValueError):
    pass


def _build(node: ast.AST) -> Any:
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, ast.Tuple):
        return tuple(_build(e) for e in node.elts)
    if isinstance(node, ast.List):
        return tuple(_build(e) for e in node.elts)
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub):
        v = _build(node.operand)
        if isinstance(v, (int, float)):
            return -v
        raise IRParseError("unary minus on a non-number")
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.UAdd):
        return _build(node.operand)
    if isinstance(node, ast.Name):
        if node.id in ("None", "True", "False"):
            return {"None": None, "True": True, "False": False}[node.id]
        if node.id in ("inf", "nan"):
            return float(node.id)
        raise IRParseError(f"bare name {node.id!r} in IR")
    if isinstance(node, ast.Call):
        if not isinstance(node.func, ast.Name):
            raise IRParseError("call through an attribute")
        fn = node.func.id
        args = [_build(a) for a in node.args]
        kwargs = {k.arg: _build(k.value) for k in node.keywords}
        if fn == "dtype":
            return NpDtype(args[0] if args else kwargs.get("dtype", ""))
        if fn == "float":
            return float(args[0])
        cls = NODE_CLASSES.get(fn)
        if cls is None:
            raise NotImplementedError(f"IR node {fn}")
        try:
            return cls(*args, **kwargs)
        except TypeError as e:
            raise IRParseError(f"bad fields for {fn}: {e}") from None
    raise IRParseError(f"unexpected syntax {type(node).__name__}")


def parse_repr(text: str) -> Any:
    """Rebuild one serialised IR object from its ``repr`` string."""
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as e:
        raise IRParseError(f"IR repr does not parse: {e}") from None
    return _build(tree.body)


# ---------------------------------------------------------------------------
# graph level
# ---------------------------------------------------------------------------

_DT_NBYTES = {"f32": 4, "f64": 8, "f16": 2, "bf16": 2, "i32": 4, "i64": 8, "u32": 4,
              "u64": 8, "i16": 2, "u16": 2, "u8": 1, "i8": 1, "bool": 1}
_DT_NP = {"f32": "float32", "f64": "float64", "f16": "float16", "bf16": "bfloat16",
          "i32": "int32", "i64": "int64", "u32": "uint32", "u64": "uint64",
          "i16": "int16", "u16": "uint16", "u8": "uint8", "i8": "int8", "bool": "bool"}


def data_type(name: str):
    """The ``DataType`` for a graph-level dtype string such as ``"f32"``."""
    return NODE_CLASSES["DataType"](name, NpDtype(_DT_NP.get(name, name)), _DT_NBYTES.get(name, 4))


@dataclasses.dataclass(frozen=True)
class TensorSpec:
    name: str
    shape: tuple
    dtype: Any


@dataclasses.dataclass(frozen=True)
class InputOp:
    pass


@dataclasses.dataclass(frozen=True)
class ConstantOp:
    name: str = ""
    value: Any = None


@dataclasses.dataclass(frozen=True)
class KernelOp:
    name: str
    body: tuple
    zero_delegated: tuple = ()
    serial: tuple = ()


@dataclasses.dataclass
class Node:
    name: str
    op: Any
    inputs: list
    outputs: list


for _c in (InputOp, ConstantOp, KernelOp):
    _c.__module__ = "emmy.compiler.graph"


class Graph:
    """Graph of InputOp / ConstantOp / KernelOp nodes (the JSON top level:
    ``inputs``, ``outputs``, ``nodes``)."""

    def __init__(self, inputs, outputs, nodes):
        self.inputs = list(inputs)
        self.outputs = list(outputs)
        self.nodes = nodes

    @classmethod
    def from_dict(cls, d: dict) -> "Graph":
        nodes = {}
        for name, nd in d["nodes"].items():
            kind = nd["op"]
            f = nd.get("op_fields", {})
            if kind == "KernelOp":
                body = tuple(parse_repr(s) if isinstance(s, str) else s for s in f.get("body", ()))
                op = KernelOp(f.get("name", name), body, tuple(f.get("zero_delegated", ()) or ()),
                              tuple(f.get("serial", ()) or ()))
            elif kind == "ConstantOp":
                op = ConstantOp(f.get("name", name), f.get("value"))
            elif kind == "InputOp":
                op = InputOp()
            else:
                raise NotImplementedError(f"graph node op {kind}")
            outs = [TensorSpec(o["name"], tuple(NODE_CLASSES["Dim"](int(s)) for s in o["shape"]),
                               data_type(o["dtype"])) for o in nd.get("outputs", ())]
            nodes[name] = Node(name, op, list(nd.get("inputs", ())), outs)
        return cls(d.get("inputs", ()), d.get("outputs", ()), nodes)


def load_graph(d: dict):
    """Deserialise with emmy-ml when it is installed, else with this reader."""
    try:  # pragma: no cover - emmy-ml is not installable offline
        from emmy.compiler.graph import Graph as EmmyGraph  # type: ignore
        if EmmyGraph is not Graph:
            return EmmyGraph.from_dict(d)
    except ImportError:
        pass
    return Graph.from_dict(d)


def load_graph_file(path) -> Any:
    with open(path) as fh:
        return load_graph(json.load(fh))


def dim(v) -> int:
    """Integer value of a ``Dim`` or plain int."""
    return int(getattr(v, "value", v))

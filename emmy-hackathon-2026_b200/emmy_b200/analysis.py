"""Structural analysis of Kernel IR bodies for the template matcher.

Index expressions in the IR are small trees of ``Var``/``Literal``/
``BinaryExpr`` (reference ``TASK.md:176-188``).  The templates need them as
affine forms ``sum(c_i * v_i) + c0`` over axis variables; anything that is not
affine (division, modulo, ternaries) makes a template decline, and the kernel
goes to the statement-by-statement lowering instead.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .ir import dim


class NotAffine(Exception):
    pass


@dataclass(frozen=True)
class Affine:
    coefs: tuple = ()          # sorted ((var, coef), ...), coef != 0
    const: int = 0

    @staticmethod
    def of(d: dict, c: int) -> "Affine":
        return Affine(tuple(sorted((k, v) for k, v in d.items() if v != 0)), int(c))

    def as_dict(self) -> dict:
        return dict(self.coefs)

    def coef(self, var: str) -> int:
        return self.as_dict().get(var, 0)

    def vars(self) -> set:
        return {k for k, _ in self.coefs}

    def __add__(self, o: "Affine") -> "Affine":
        d = self.as_dict()
        for k, v in o.coefs:
            d[k] = d.get(k, 0) + v
        return Affine.of(d, self.const + o.const)

    def __sub__(self, o: "Affine") -> "Affine":
        return self + o.scale(-1)

    def scale(self, s: int) -> "Affine":
        return Affine.of({k: v * s for k, v in self.coefs}, self.const * s)

    def is_const(self) -> bool:
        return not self.coefs


def affine(e, env: dict | None = None) -> Affine:
    """Affine form of an integer index expression, or raise :class:`NotAffine`.

    ``env`` maps names bound by ``Let`` (or template-chosen substitutions) to
    their affine forms."""
    env = env or {}
    k = type(e).__name__
    if isinstance(e, int) and not isinstance(e, bool):
        return Affine((), e)
    if k == "Literal":
        if isinstance(e.value, bool) or not isinstance(e.value, int):
            raise NotAffine("non-integer literal")
        return Affine((), e.value)
    if k == "Var":
        if e.name in env:
            return env[e.name]
        return Affine(((e.name, 1),), 0)
    if k == "BinaryExpr":
        if e.op == "+":
            return affine(e.left, env) + affine(e.right, env)
        if e.op == "-":
            return affine(e.left, env) - affine(e.right, env)
        if e.op == "*":
            a, b = affine(e.left, env), affine(e.right, env)
            if a.is_const():
                return b.scale(a.const)
            if b.is_const():
                return a.scale(b.const)
            raise NotAffine("product of variables")
    raise NotAffine(f"{k} {getattr(e, 'op', '')}")


def flat_index(index: tuple, shape: tuple, env: dict | None = None) -> Affine:
    """Row-major flat element offset of a multi-dimensional index (the
    reference linearises the same way, ``compile.py:590-598``)."""
    if len(index) == 0:
        return Affine((), 0)
    if len(index) != len(shape):
        raise NotAffine("index rank does not match buffer rank")
    out = Affine((), 0)
    stride = 1
    for ix, ext in zip(reversed(index), reversed(shape)):
        out = out + affine(ix, env).scale(stride)
        stride *= ext
    return out


def kind(s) -> str:
    return type(s).__name__


def walk(stmts):
    """All statements of a body, depth first."""
    for s in stmts:
        yield s
        for attr in ("body", "else_body"):
            sub = getattr(s, attr, None)
            if isinstance(sub, tuple):
                yield from walk(sub)


def axis_extents(tile) -> list[tuple[str, int]]:
    return [(a.name, dim(a.extent)) for a in tile.axes]


def is_lit(e, value=None) -> bool:
    return kind(e) == "Literal" and (value is None or e.value == value)


def cond_var_eq(cond, var: str, value: int = 0) -> bool:
    """``cond`` is ``(var == value)``."""
    return (kind(cond) == "BinaryExpr" and cond.op == "==" and kind(cond.left) == "Var"
            and cond.left.name == var and is_lit(cond.right, value))


@dataclass
class Buffers:
    """Shapes and dtypes of every tensor in the graph, plus meta facts."""
    shapes: dict = field(default_factory=dict)
    dtypes: dict = field(default_factory=dict)
    constants: dict = field(default_factory=dict)   # ConstantOp name -> value

    def size(self, name: str) -> int:
        n = 1
        for d in self.shapes[name]:
            n *= d
        return n

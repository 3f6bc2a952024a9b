"""Elementwise operations of the Kernel IR, emitted as sm_100a PTX.

The IR names each operation by its Emmy ``ElementwiseImpl`` name (the
reference's dispatch tables are at ``compile.py:667-731``).  Arithmetic that
must match numpy bit for bit (pointwise kernels) uses the ``.rn`` forms,
which ptxas never contracts into FMAs; reductions and fused row kernels use
the same instructions, so a template and the generic lowering agree.

Transcendentals are written from their mathematical definitions:

* ``exp(x) = 2^(x*log2 e)`` with the product split into ``t + r`` (``t`` the
  f32-rounded product, ``r`` its exact FMA residual plus ``x`` times the tail
  of log2 e), evaluated as ``ex2.approx(t) * (1 + r ln 2)``.  ``|r| <= 2^-24|t|``,
  so the first-order correction leaves an error far below one f32 ulp on top
  of ``ex2.approx``'s own;
* ``sqrt``/``reciprocal`` are the correctly rounded ``sqrt.rn``/``rcp.rn``;
  ``rsqrt`` is ``rcp.rn(sqrt.rn(x))`` as in the reference (``compile.py:784-787``);
* ``log(x) = lg2.approx(x) * ln 2``; ``tanh``, ``sigmoid``, ``silu`` from ``exp``.
"""
from __future__ import annotations

import math

from .ptx import Kernel, f32_hex

LOG2E_HI = 1.4426950216293335  # float32(log2 e)
LOG2E_LO = math.log2(math.e) - LOG2E_HI
LN2 = math.log(2.0)

BINARY = {"add", "subtract", "multiply", "divide", "maximum", "minimum", "pow", "mod",
          "remainder", "fmod", "floor_divide", "equal", "not_equal", "greater",
          "greater_equal", "less", "less_equal"}


class UnsupportedOp(NotImplementedError):
    pass


def _f(v) -> str:
    """A register or an f32 immediate."""
    if isinstance(v, (int, float)):
        return f32_hex(v)
    return v


def emit_exp2_scaled(k: Kernel, x: str, scale_hi: float, scale_lo: float) -> str:
    """``2^(x*(scale_hi+scale_lo))`` with the compensated product described in
    the module docstring."""
    t = k.reg("f")
    k(f"mul.rn.f32 {t}, {x}, {f32_hex(scale_hi)};")
    r = k.reg("f")
    k(f"neg.f32 {r}, {t};")
    k(f"fma.rn.f32 {r}, {x}, {f32_hex(scale_hi)}, {r};")
    k(f"fma.rn.f32 {r}, {x}, {f32_hex(scale_lo)}, {r};")
    p = k.reg("f")
    k(f"ex2.approx.f32 {p}, {t};")
    q = k.reg("f")
    k(f"mul.rn.f32 {q}, {r}, {f32_hex(LN2)};")
    out = k.reg("f")
    k(f"fma.rn.f32 {out}, {p}, {q}, {p};")
    return out


def emit_exp(k: Kernel, x: str) -> str:
    return emit_exp2_scaled(k, x, LOG2E_HI, LOG2E_LO)


def emit_op_f32(k: Kernel, op: str, args: list) -> str:
    """Emit one f32 elementwise op; returns the destination register."""
    a = [_f(x) for x in args]
    d = k.reg("f")
    if op == "add":
        k(f"add.rn.f32 {d}, {a[0]}, {a[1]};")
    elif op == "subtract":
        k(f"sub.rn.f32 {d}, {a[0]}, {a[1]};")
    elif op == "multiply":
        k(f"mul.rn.f32 {d}, {a[0]}, {a[1]};")
    elif op == "divide":
        k(f"div.rn.f32 {d}, {a[0]}, {a[1]};")
    elif op in ("fma", "mul_add"):
        k(f"fma.rn.f32 {d}, {a[0]}, {a[1]}, {a[2]};")
    elif op == "maximum":
        k(f"max.f32 {d}, {a[0]}, {a[1]};")
    elif op == "minimum":
        k(f"min.f32 {d}, {a[0]}, {a[1]};")
    elif op in ("copy", "pad"):
        k(f"mov.f32 {d}, {a[0]};")
    elif op in ("neg", "negative"):
        k(f"neg.f32 {d}, {a[0]};")
    elif op in ("abs", "fabs"):
        k(f"abs.f32 {d}, {a[0]};")
    elif op == "relu":
        k(f"max.f32 {d}, {a[0]}, 0f00000000;")
    elif op == "square":
        k(f"mul.rn.f32 {d}, {a[0]}, {a[0]};")
    elif op == "reciprocal":
        k(f"rcp.rn.f32 {d}, {a[0]};")
    elif op == "sqrt":
        k(f"sqrt.rn.f32 {d}, {a[0]};")
    elif op == "rsqrt":
        s = k.reg("f")
        k(f"sqrt.rn.f32 {s}, {a[0]};")
        k(f"rcp.rn.f32 {d}, {s};")
    elif op in ("exp", "exp_fast"):
        return emit_exp(k, a[0])
    elif op == "exp2":
        k(f"ex2.approx.f32 {d}, {a[0]};")
    elif op in ("log", "log2"):
        l2 = k.reg("f")
        k(f"lg2.approx.f32 {l2}, {a[0]};")
        if op == "log2":
            return l2
        k(f"mul.rn.f32 {d}, {l2}, {f32_hex(LN2)};")
    elif op == "sigmoid":
        n = k.reg("f")
        k(f"neg.f32 {n}, {a[0]};")
        e = emit_exp(k, n)
        s = k.reg("f")
        k(f"add.rn.f32 {s}, {e}, 0f3F800000;")
        k(f"rcp.rn.f32 {d}, {s};")
    elif op == "silu":
        n = k.reg("f")
        k(f"neg.f32 {n}, {a[0]};")
        e = emit_exp(k, n)
        s = k.reg("f")
        k(f"add.rn.f32 {s}, {e}, 0f3F800000;")
        k(f"div.rn.f32 {d}, {a[0]}, {s};")
    elif op == "tanh":
        # tanh x = 1 - 2 / (exp(2x) + 1), saturating correctly at both ends
        x2 = k.reg("f")
        k(f"add.rn.f32 {x2}, {a[0]}, {a[0]};")
        e = emit_exp(k, x2)
        s = k.reg("f")
        k(f"add.rn.f32 {s}, {e}, 0f3F800000;")
        q = k.reg("f")
        k(f"div.rn.f32 {q}, 0f40000000, {s};")
        k(f"sub.rn.f32 {d}, 0f3F800000, {q};")
    elif op in ("floor", "ceil", "trunc", "round"):
        mode = {"floor": "rmi", "ceil": "rpi", "trunc": "rzi", "round": "rni"}[op]
        k(f"cvt.{mode}.f32.f32 {d}, {a[0]};")
    else:
        raise UnsupportedOp(f"elementwise op {op} (f32)")
    return d


def identity_f32(op: str) -> float:
    """Start value of a reduce accumulator (reference ``compile.py:576-583``:
    maximum starts at -1e30, minimum at 1e30)."""
    return {"add": 0.0, "multiply": 1.0, "maximum": -1e30, "minimum": 1e30}[op]

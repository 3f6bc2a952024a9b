"""Pieces shared by the sm_100a kernel templates.

A template owns the memory schedule and the parallel structure of a kernel
(which thread touches which bytes, how partial results combine); the IR owns
the arithmetic.  :class:`Chain` executes the IR's own ``Let``/``Assign``/
``Accum`` statements on PTX registers, in IR order, so a template computes
exactly the operations the IR names (reference statement semantics:
``stmt_assign`` ``compile.py:1273-1286``, ``stmt_accum`` ``:1606-1610``,
``stmt_let`` ``:1388-1410``).  Loads are resolved by a template callback,
because *where* a value comes from (a vector register, shared memory, a
hoisted constant) is the template's business.
"""
from __future__ import annotations

from ..analysis import kind
from ..ops import emit_op_f32, identity_f32
from ..ptx import Kernel, f32_hex


class TemplateMismatch(Exception):
    """The IR does not have the shape a template handles."""


def dtype_name(dt) -> str | None:
    if dt is None:
        return None
    return getattr(dt, "name", dt)


class Chain:
    def __init__(self, k: Kernel, env: dict, load):
        self.k = k
        self.env = env          # IR name -> PTX register or python float
        self.load = load        # callback(Load stmt) -> list of registers

    def value(self, name: str) -> str:
        v = self.env[name]
        if isinstance(v, (int, float)):
            return f32_hex(v)
        return v

    def run(self, stmts) -> None:
        for s in stmts:
            self.stmt(s)

    def stmt(self, s) -> None:
        k = kind(s)
        if k == "Let":
            v = s.value
            if kind(v) != "Literal":
                raise TemplateMismatch(f"Let of {kind(v)}")
            self.env[s.name] = float(v.value)
        elif k == "Load":
            regs = self.load(s)
            for n, r in zip(s.names, regs):
                self.env[n] = r
        elif k == "Assign":
            ty = dtype_name(s.dtype)
            if ty not in (None, "f32"):
                raise TemplateMismatch(f"Assign dtype {ty}")
            args = [self.value(a) for a in s.args]
            self.env[s.name] = emit_op_f32(self.k, s.op.name, args)
        elif k == "Accum":
            acc = self.env[s.name]
            left = self.value(s.base) if s.base else acc
            r = emit_op_f32(self.k, s.op.name, [left, self.value(s.value)])
            self.k(f"mov.f32 {acc}, {r};")
        elif k == "Init":
            r = self.k.reg("f")
            self.k(f"mov.f32 {r}, {f32_hex(float(s.identity))};")
            self.env[s.name] = r
        else:
            raise TemplateMismatch(f"statement {k} in an arithmetic chain")


def accum_identity(op: str) -> float:
    return identity_f32(op)


def linear_ids(k: Kernel, grid, block):
    """Linear thread id inside the CTA, linear CTA id, and the flat global id,
    as the reference derives them (``compile.py:2339-2388``)."""
    bx, by, bz = block
    gx, gy, gz = grid
    tid = k.special("%tid.x")
    if by * bz > 1:
        ty = k.special("%tid.y")
        t = k.reg("r")
        k(f"mad.lo.s32 {t}, {ty}, {bx}, {tid};")
        tid = t
        if bz > 1:
            tz = k.special("%tid.z")
            t2 = k.reg("r")
            k(f"mad.lo.s32 {t2}, {tz}, {bx * by}, {tid};")
            tid = t2
    cta = k.special("%ctaid.x")
    if gy * gz > 1:
        cy = k.special("%ctaid.y")
        c = k.reg("r")
        k(f"mad.lo.s32 {c}, {cy}, {gx}, {cta};")
        cta = c
        if gz > 1:
            cz = k.special("%ctaid.z")
            c2 = k.reg("r")
            k(f"mad.lo.s32 {c2}, {cz}, {gx * gy}, {cta};")
            cta = c2
    gid = k.reg("r")
    k(f"mad.lo.s32 {gid}, {cta}, {bx * by * bz}, {tid};")
    return tid, cta, gid


def vec_suffix(v: int) -> str:
    return "" if v == 1 else f".v{v}"


def reg_list(regs) -> str:
    return "{" + ", ".join(regs) + "}" if len(regs) > 1 else regs[0]


def ld_global_f32(k: Kernel, addr: str, v: int, *, nc: bool = True, hint: str = "") -> list:
    regs = k.regs("f", v)
    space = "global.nc" if nc else "global"
    k(f"ld.{space}{hint}{vec_suffix(v)}.f32 {reg_list(regs)}, [{addr}];")
    return regs


def st_global_f32(k: Kernel, addr: str, regs, hint: str = "", pred: str | None = None) -> None:
    guard = f"@{pred} " if pred else ""
    k(f"{guard}st.global{hint}{vec_suffix(len(regs))}.f32 [{addr}], {reg_list(regs)};")


def addr_of(k: Kernel, base: str, elem_index_reg: str, nbytes: int = 4) -> str:
    """``base + index * nbytes`` as a 64-bit address (index is a 32-bit reg)."""
    off = k.reg("rd")
    k(f"mul.wide.u32 {off}, {elem_index_reg}, {nbytes};")
    a = k.reg("rd")
    k(f"add.s64 {a}, {base}, {off};")
    return a


def pick_vec(n: int, per: int, maxv: int = 8) -> int:
    """Largest vector width v <= maxv (power of two) with n % (v*per) == 0."""
    v = maxv
    while v > 1 and n % (v * per):
        v //= 2
    return v

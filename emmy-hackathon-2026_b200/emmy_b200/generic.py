"""Statement-by-statement sm_100a lowering for IRs no template accepts.

This is the drop-in safety net: every Kernel IR statement the reference
compiler handles (its dispatch, ``compile.py:2579-2616``) is lowered here in
IR order, one PTX sequence per statement, with the reference's semantics:

* launch decode -- flat thread id = CTA-linear * threads + thread-linear,
  cells decoded row-major over the Tile axes (grouped rasterisation and
  auxiliary producer threads as in ``compile.py:2390-2534``), the bound guard
  ``gid < cells`` derived from the Tile (not in the IR, ``TASK.md:229``), and
  the specials ``lane = tid.x & 31``, ``warp = tid.x >> 5``;
* values -- narrow floats load as b16 and compute in f32; narrow integers
  compute in 32 bits; a store converts to the buffer's dtype with C
  semantics; ``Accum`` folds into an accumulator that a seeded loop
  initialises to the op's identity before the loop (``compile.py:2024-2046``);
* shared memory -- static arrays, or one dynamic pool ``__emmy_smem`` when
  meta gives ``smem_bytes``; ``WarpShuffle`` is an XOR butterfly over the
  active lanes; ``TreeHalve`` halves a power-of-two tree in shared memory with
  a barrier per level and broadcasts the root;
* ``Sync``: barrier 0 is CTA-wide (its count is ignored, as Emmy renders
  ``__syncthreads()``), named barriers take their count, ``warp`` syncs the warp.

Loops with a static trip count of at most ``UNROLL_CAP`` and no nested loop
are unrolled, the loop variable bound to each constant in turn, and an f32
``multiply`` whose only use is the next statement's ``Accum`` add becomes one
``fma.rn.f32`` -- the reference's own two speed rules (``compile.py:1882-1928``,
``2244-2264``); every other loop stays a plain loop, and memory accesses are
scalar: correctness first; the templates are the fast paths.
"""
from __future__ import annotations

import math
import struct
from math import prod

from .analysis import kind, walk
from .fragments import FragmentLowering
from .wgmma import WgmmaLowering
from .ir import dim
from .ops import LN2, UnsupportedOp, emit_exp, emit_op_f32, identity_f32
from .ptx import PARAM_TYPES, Kernel, f32_hex, f64_hex

INT_TYPES = {"i32", "i64", "u32", "u64", "bool", "u8", "u16", "i16", "i8"}
WIDEN = {"f16", "bf16"}
NBYTES = {"f32": 4, "f64": 8, "f16": 2, "bf16": 2, "i32": 4, "i64": 8, "u32": 4, "u64": 8,
          "u8": 1, "i8": 1, "u16": 2, "i16": 2, "bool": 1}
REG = {"f32": "f", "f64": "fd", "i32": "r", "u32": "r", "i64": "rd", "u64": "rd", "bool": "r"}
MOVTY = {"f": "f32", "fd": "f64", "r": "b32", "rd": "b64", "h": "b16"}
PTY = {"f32": "f32", "f64": "f64", "i32": "s32", "u32": "u32", "i64": "s64", "u64": "u64",
       "bool": "u32"}
LDTY = {"f32": "f32", "f64": "f64", "i32": "s32", "u32": "u32", "i64": "s64", "u64": "u64",
        "u8": "u8", "i8": "s8", "u16": "u16", "i16": "s16", "bool": "u8"}
SMEM_TY = {"float": "f32", "float32": "f32", "double": "f64", "float64": "f64", "half": "f16",
           "__half": "f16", "float16": "f16", "bfloat16": "bf16", "__nv_bfloat16": "bf16",
           "int": "i32", "int32": "i32", "int32_t": "i32", "unsigned int": "u32",
           "uint32_t": "u32", "long long": "i64", "int64_t": "i64",
           "unsigned long long": "u64", "uint64_t": "u64", "char": "i8", "signed char": "i8",
           "uint8_t": "u8", "int8_t": "i8", "short": "i16", "int16_t": "i16",
           "unsigned short": "u16", "uint16_t": "u16", "bool": "bool"}
CMP = {"equal": "eq", "not_equal": "ne", "greater": "gt", "greater_equal": "ge",
       "less": "lt", "less_equal": "le"}
BUILTINS = {"thread_idx.x": "%tid.x", "thread_idx.y": "%tid.y", "thread_idx.z": "%tid.z",
            "threadIdx.x": "%tid.x", "threadIdx.y": "%tid.y", "threadIdx.z": "%tid.z",
            "block_idx.x": "%ctaid.x", "block_idx.y": "%ctaid.y", "block_idx.z": "%ctaid.z",
            "blockIdx.x": "%ctaid.x", "blockIdx.y": "%ctaid.y", "blockIdx.z": "%ctaid.z",
            "block_dim.x": "%ntid.x", "blockDim.x": "%ntid.x", "lane_id": "%laneid"}


def _calc_ty(ty: str) -> str:
    """The type a value of dtype ``ty`` is computed in."""
    if ty in WIDEN:
        return "f32"
    if ty in ("u8", "u16"):
        return "u32"
    if ty in ("i8", "i16"):
        return "i32"
    return ty


class GenericLowering(FragmentLowering, WgmmaLowering):
    name = "generic"

    def __init__(self, ctx):
        self.ctx = ctx
        if ctx.tile is None:
            raise NotImplementedError("expected a single Tile at top level")

    # ------------------------------------------------------------------ setup
    def emit(self) -> str:
        ctx = self.ctx
        self.k = k = Kernel(ctx.entry, ctx.params())
        k.comment("emmy-b200 generic lowering")
        self.vals = {}       # SSA name -> (operand, type)
        self.ints = {}       # int name (axis, Let) -> operand (s32 register or immediate)
        self.base = {}       # global buffer -> 64-bit address register
        self.smem = {}       # smem name -> dict(extents, ty, nbytes, off | symbol)
        self.dynamic = ctx.smem_bytes > 0
        self.smem_used = 0
        self.max_align = 16
        for a in ctx.arg_order:
            if a in ctx.scalar_tys:
                ty = ctx.scalar_tys[a]
                cty = _calc_ty(ty)
                r = k.reg(REG.get(cty, "r"))
                pty = PARAM_TYPES.get(ty, "u32")
                if ty in ("f16", "bf16"):
                    h = k.reg("h")
                    k(f"ld.param.b16 {h}, [param_{a}];")
                    k(f"cvt.f32.{ty} {r}, {h};")
                elif ty in ("u8", "bool", "u16", "i16"):
                    k(f"ld.param.{pty} {r}, [param_{a}];")
                else:
                    k(f"ld.param.{pty} {r}, [param_{a}];")
                if cty in INT_TYPES:
                    self.ints[a] = r
                self.vals[a] = (r, cty)
            else:
                self.base[a] = k.param_ptr(a)
        self.tmaps = {}      # TmaDescriptor name -> (param address register, info)
        self.cells = {}      # (carrier, index) -> [state register, next register, type]
        self._declare_mbarriers(ctx.tile)
        self.compile_tile(ctx.tile)
        k("ret;")
        if self.dynamic:
            if self.smem_used > ctx.smem_bytes:
                raise NotImplementedError(
                    f"smem layout {self.smem_used} exceeds meta smem_bytes {ctx.smem_bytes}")
            k.decl(f".extern .shared .align {self.max_align} .b8 __emmy_smem[];")
        return k.render()

    def compile_tile(self, tile):
        k, ctx = self.k, self.ctx
        extents = [dim(a.extent) for a in tile.axes]
        ncells = prod(extents)
        total = ctx.total_threads
        if ncells > total:
            raise NotImplementedError("fewer threads than cells")
        bx, by, bz = ctx.block
        gx, gy, gz = ctx.grid
        tid = k.special("%tid.x")
        self.tid_x = tid
        tlin = tid
        if by * bz > 1:
            ty = k.special("%tid.y")
            t = k.reg("r")
            k(f"mad.lo.s32 {t}, {ty}, {bx}, {tlin};")
            tlin = t
            if bz > 1:
                tz = k.special("%tid.z")
                t2 = k.reg("r")
                k(f"mad.lo.s32 {t2}, {tz}, {bx * by}, {tlin};")
                tlin = t2
        clin = k.special("%ctaid.x")
        if gy * gz > 1:
            cy = k.special("%ctaid.y")
            c = k.reg("r")
            k(f"mad.lo.s32 {c}, {cy}, {gx}, {clin};")
            clin = c
            if gz > 1:
                cz = k.special("%ctaid.z")
                c2 = k.reg("r")
                k(f"mad.lo.s32 {c2}, {cz}, {gx * gy}, {clin};")
                clin = c2
        threads = bx * by * bz
        # 64-bit flat cell id (cells can exceed 2^31)
        gid64 = k.reg("rd")
        k(f"mul.wide.u32 {gid64}, {clin}, {threads};")
        t64 = k.reg("rd")
        k(f"cvt.u64.u32 {t64}, {tlin};")
        k(f"add.s64 {gid64}, {gid64}, {t64};")
        lane = k.reg("r")
        k(f"and.b32 {lane}, {tid}, 31;")
        warp = k.reg("r")
        k(f"shr.u32 {warp}, {tid}, 5;")
        self.ints["lane"] = lane
        self.ints["warp"] = warp
        self.builtin_warp = warp
        aux = int(getattr(tile, "aux_threads", 0) or 0)
        if aux:
            bt = int(tile.block_threads)
            w = k.reg("r")
            k(f"rem.u32 {w}, {tlin}, {bt};")
            k(f"mul.wide.u32 {gid64}, {clin}, {bt};")
            w64 = k.reg("rd")
            k(f"cvt.u64.u32 {w64}, {w};")
            k(f"add.s64 {gid64}, {gid64}, {w64};")
        done = k.label("DONE")
        if ncells < total or aux:
            p = k.reg("p")
            k(f"setp.ge.u64 {p}, {gid64}, {ncells};")
            k(f"@{p} bra {done};")
        self.gid64 = gid64
        cell = gid64
        if ctx.total_threads < 2 ** 31:
            # every cell id fits in 32 bits: decode with 32-bit integer ops
            # (a 64-bit divide or remainder is a long emulated sequence)
            cell = k.reg("r")
            k(f"cvt.u32.u64 {cell}, {gid64};")
        self._wg_begin(tile)
        self.decode(tile, cell, extents)
        self.body(tile.body)
        k.mark(done)
        self._wg_end()

    def decode(self, tile, gid64, extents):
        """Row-major decode of the flat cell id over the Tile axes, with
        Emmy's grouped rasterisation of two adjacent block axes.  ``gid64``
        is a 64-bit register, or a 32-bit one when every cell id fits
        (then power-of-two strides and extents decode by shift and mask)."""
        k = self.k
        wide = gid64.startswith("%rd")

        def divide(dst, src, d):
            if not wide and d & (d - 1) == 0:
                k(f"shr.u32 {dst}, {src}, {d.bit_length() - 1};")
            else:
                k(f"div.u{64 if wide else 32} {dst}, {src}, {d};")

        def modulo(dst, src, d):
            if not wide and d & (d - 1) == 0:
                k(f"and.b32 {dst}, {src}, {d - 1};")
            else:
                k(f"rem.u{64 if wide else 32} {dst}, {src}, {d};")
        strides = [1] * len(extents)
        acc = 1
        for i in range(len(extents) - 1, -1, -1):
            strides[i] = acc
            acc *= extents[i]
        names = [a.name for a in tile.axes]
        raster = None
        rg, ra = getattr(tile, "raster_group", None), getattr(tile, "raster_axes", None)
        if rg and ra and ra[0] in names and ra[1] in names:
            mi, ni = names.index(ra[0]), names.index(ra[1])
            if ni == mi + 1:
                gi, oi = (mi, ni) if getattr(tile, "raster_orient", "m") == "m" else (ni, mi)
                g = min(rg, extents[gi])
                if extents[gi] > 1 and g > 1:
                    raster = (gi, oi, g)
        for i, name in enumerate(names):
            if extents[i] == 1:
                self.ints[name] = "0"
                continue
            q = k.reg("rd" if wide else "r")
            if strides[i] != 1:
                divide(q, gid64, strides[i])
            else:
                k(f"mov.{'u64' if wide else 'u32'} {q}, {gid64};")
            if i != 0:
                modulo(q, q, extents[i])
            if wide:
                r = k.reg("r")
                k(f"cvt.u32.u64 {r}, {q};")
            else:
                r = q
            self.ints[name] = r
        if raster is not None:
            gi, oi, g = raster
            mi, ni = min(gi, oi), max(gi, oi)
            ea, eb = extents[gi], extents[oi]
            sub = k.reg("rd" if wide else "r")
            divide(sub, gid64, strides[ni])
            if mi != 0:
                modulo(sub, sub, ea * eb)
            if wide:
                s32 = k.reg("r")
                k(f"cvt.u32.u64 {s32}, {sub};")
            else:
                s32 = sub
            grp = k.reg("r")
            k(f"div.u32 {grp}, {s32}, {g * eb};")
            rem = k.reg("r")
            k(f"rem.u32 {rem}, {s32}, {g * eb};")
            gsz = k.reg("r")
            k(f"mul.lo.u32 {gsz}, {grp}, {g};")
            left = k.reg("r")
            k(f"sub.u32 {left}, {ea}, {gsz};")
            k(f"min.u32 {left}, {left}, {g};")
            a_ = k.reg("r")
            k(f"rem.u32 {a_}, {rem}, {left};")
            k(f"add.u32 {a_}, {a_}, {gsz};")
            b_ = k.reg("r")
            k(f"div.u32 {b_}, {rem}, {left};")
            self.ints[names[gi]] = a_
            self.ints[names[oi]] = b_

    # --------------------------------------------------------- expressions
    def ival(self, e) -> str:
        """An integer index expression as a 32-bit operand."""
        k = self.k
        t = kind(e)
        if isinstance(e, int):
            return str(e)
        if t == "Literal":
            if isinstance(e.value, float) and not float(e.value).is_integer():
                raise NotImplementedError("float literal in an index")
            return str(int(e.value))
        if t == "Var":
            if e.name in self.ints:
                return self.ints[e.name]
            if e.name in self.vals:
                v, ty = self.vals[e.name]
                if ty in ("i32", "u32", "bool"):
                    return v
                r = k.reg("r")
                if ty in ("i64", "u64"):
                    k(f"cvt.u32.u64 {r}, {v};")
                else:
                    k(f"cvt.rzi.s32.{ty} {r}, {v};")
                return r
            raise NotImplementedError(f"unknown index variable {e.name}")
        if t == "Builtin":
            sreg = BUILTINS.get(e.name)
            if sreg is None:
                raise NotImplementedError(f"builtin {e.name}")
            return k.special(sreg)
        if t == "CastExpr":
            return self.ival(e.expr)
        if t == "TernaryExpr":
            p = self.pred(e.cond)
            a, b = self.ival(e.if_true), self.ival(e.if_false)
            r = k.reg("r")
            k(f"selp.b32 {r}, {a}, {b}, {p};")
            return r
        if t == "FlatIndex":
            return self.flat(e.index, self.shape_of(e.buffer))
        if t == "BinaryExpr":
            if e.op in ("<", "<=", ">", ">=", "==", "!=", "&&", "||"):
                p = self.pred(e)
                r = k.reg("r")
                k(f"selp.u32 {r}, 1, 0, {p};")
                return r
            a, b = self.ival(e.left), self.ival(e.right)
            if _is_imm(a) and _is_imm(b):
                return str(_fold(e.op, int(a), int(b)))
            op = {"+": "add.s32", "-": "sub.s32", "*": "mul.lo.s32", "/": "div.s32",
                  "//": "div.s32", "%": "rem.s32", "<<": "shl.b32", ">>": "shr.s32", "&": "and.b32",
                  "|": "or.b32", "^": "xor.b32", "min": "min.s32", "max": "max.s32"}.get(e.op)
            if op is None:
                raise NotImplementedError(f"index operator {e.op}")
            if e.op == "+" and a == "0":
                return b
            if e.op in ("+", "-") and b == "0":
                return a
            if e.op == "*" and b == "1":
                return a
            if e.op == "*" and a == "1":
                return b
            r = k.reg("r")
            if _is_imm(a):
                if e.op in ("+", "*", "&", "|", "^", "min", "max"):
                    a, b = b, a
                else:
                    t2 = k.reg("r")
                    k(f"mov.b32 {t2}, {a};")
                    a = t2
            k(f"{op} {r}, {a}, {b};")
            return r
        raise NotImplementedError(f"index expression {t}")

    def pred(self, e) -> str:
        k = self.k
        t = kind(e)
        if t == "BinaryExpr" and e.op in ("&&", "||"):
            a, b = self.pred(e.left), self.pred(e.right)
            p = k.reg("p")
            k(f"{'and' if e.op == '&&' else 'or'}.pred {p}, {a}, {b};")
            return p
        if t == "BinaryExpr" and e.op in ("==", "!=", "<", "<=", ">", ">="):
            cmp = {"==": "eq", "!=": "ne", "<": "lt", "<=": "le", ">": "gt", ">=": "ge"}[e.op]
            fl = self._float_side(e.left) or self._float_side(e.right)
            p = k.reg("p")
            if fl:
                ty = fl
                a, b = self.fval(e.left, ty), self.fval(e.right, ty)
                k(f"setp.{cmp}.{ty} {p}, {a}, {b};")
            else:
                a, b = self.ival(e.left), self.ival(e.right)
                if _is_imm(a):
                    t2 = k.reg("r")
                    k(f"mov.b32 {t2}, {a};")
                    a = t2
                k(f"setp.{cmp}.s32 {p}, {a}, {b};")
            return p
        # a value used as a predicate: non-zero
        v = self.ival(e)
        p = k.reg("p")
        k(f"setp.ne.s32 {p}, {v}, 0;")
        return p

    def _float_side(self, e):
        t = kind(e)
        if t == "Var" and e.name in self.vals and self.vals[e.name][1] in ("f32", "f64"):
            return self.vals[e.name][1]
        if t == "Literal" and isinstance(e.value, float) and not float(e.value).is_integer():
            return "f32"
        return None

    def fval(self, e, ty) -> str:
        t = kind(e)
        if t == "Literal":
            return f32_hex(float(e.value)) if ty == "f32" else f64_hex(float(e.value))
        if t == "Var" and e.name in self.vals:
            v, vty = self.vals[e.name]
            return self.convert(v, vty, ty)
        v = self.ival(e)
        r = self.k.reg(REG[ty])
        self.k(f"cvt.rn.{ty}.s32 {r}, {v};")
        return r

    def shape_of(self, buf):
        if buf in self.smem:
            return self.smem[buf]["extents"]
        return self.ctx.bufs.shapes.get(buf, ())

    def flat(self, index, shape) -> str:
        """Row-major flat element index (reference ``compile.py:559-571``)."""
        if not index:
            return "0"
        if len(index) == 1:
            return self.ival(index[0])
        acc = "0"
        for i, e in enumerate(index):
            suffix = prod(shape[i + 1:]) if i + 1 < len(shape) else 1
            term = self.ival(e)
            if suffix != 1:
                term = self._imul(term, suffix)
            acc = self._iadd(acc, term)
        return acc

    def _imul(self, a, c):
        if _is_imm(a):
            return str(int(a) * c)
        r = self.k.reg("r")
        self.k(f"mul.lo.s32 {r}, {a}, {c};")
        return r

    def _iadd(self, a, b):
        if _is_imm(a) and _is_imm(b):
            return str(int(a) + int(b))
        if a == "0":
            return b
        if b == "0":
            return a
        if _is_imm(a):
            a, b = b, a
        r = self.k.reg("r")
        self.k(f"add.s32 {r}, {a}, {b};")
        return r

    # --------------------------------------------------------- addressing
    def gaddr(self, buf, flat, nbytes) -> str:
        k = self.k
        if _is_imm(flat):
            a = k.reg("rd")
            k(f"add.s64 {a}, {self.base[buf]}, {int(flat) * nbytes};")
            return a
        off = k.reg("rd")
        k(f"mul.wide.s32 {off}, {flat}, {nbytes};")
        a = k.reg("rd")
        k(f"add.s64 {a}, {self.base[buf]}, {off};")
        return a

    def saddr(self, buf, flat) -> str:
        k = self.k
        info = self.smem[buf]
        base = k.reg("r")
        if self.dynamic:
            k(f"mov.u32 {base}, __emmy_smem;")
            if info["off"]:
                k(f"add.u32 {base}, {base}, {info['off']};")
        else:
            k(f"mov.u32 {base}, {info['sym']};")
        if _is_imm(flat):
            if int(flat):
                k(f"add.u32 {base}, {base}, {int(flat) * info['nbytes']};")
            return base
        a = k.reg("r")
        k(f"mad.lo.s32 {a}, {flat}, {info['nbytes']}, {base};")
        return a

    # --------------------------------------------------------- statements
    def body(self, stmts):
        stmts = list(stmts)
        uses = self._uses(stmts)
        i = 0
        while i < len(stmts):
            s = stmts[i]
            nxt = stmts[i + 1] if i + 1 < len(stmts) else None
            if (kind(s) == "Assign" and s.op.name == "multiply" and len(s.args) == 2
                    and uses.get(s.name, 0) == 1 and nxt is not None
                    and kind(nxt) == "Accum" and nxt.value == s.name and nxt.op.name == "add"
                    and (nxt.dtype is None or nxt.dtype.name == "f32")
                    and all(self.vals.get(a, (None, ""))[1] == "f32" for a in s.args)):
                # acc = acc + a*b in one rounding, as the reference contracts it
                reg, ty = self.accum_reg(nxt)
                if ty == "f32":
                    left = self.vals[nxt.base][0] if nxt.base else reg
                    a, b = (self.vals[x][0] for x in s.args)
                    self.k(f"fma.rn.f32 {reg}, {a}, {b}, {left};")
                    self.vals[nxt.name] = (reg, ty)
                    i += 2
                    continue
            if isinstance(s, _StepMark):
                self._step(s.cells, s.begin)
            else:
                getattr(self, "s_" + kind(s), self.s_unsupported)(s)
            i += 1

    @staticmethod
    def _uses(stmts) -> dict:
        """How often each name is read in ``stmts`` (nested bodies included):
        operand names of statements and variables of their expressions
        (conditions, indices, loop bounds)."""
        out: dict = {}

        def count(n):
            out[n] = out.get(n, 0) + 1

        def expr(e):
            if e is None or isinstance(e, (int, float)):
                return
            if isinstance(e, tuple):
                for x in e:
                    expr(x)
                return
            fv = getattr(e, "free_vars", None)
            if fv is not None:
                for n in fv():
                    count(n)
        for st in walk(stmts):
            for a in getattr(st, "args", ()) or ():
                if isinstance(a, str):
                    count(a)
                else:
                    expr(a)
            for f in ("value", "base"):
                v = getattr(st, f, None)
                if isinstance(v, str):
                    count(v)
                else:
                    expr(v)
            for v in getattr(st, "values", ()) or ():
                if isinstance(v, str):
                    count(v)
            for f in ("cond", "index", "src_index", "smem_index", "start", "step", "end"):
                expr(getattr(st, f, None))
        return out

    def s_unsupported(self, s):
        raise NotImplementedError(f"statement {kind(s)}")

    def load_ty(self, s):
        if s.dtype is not None:
            return s.dtype.name
        if s.input in self.smem:
            return self.smem[s.input]["ty"]
        return self.ctx.bufs.dtypes.get(s.input, "f32")

    def s_Load(self, s):
        k = self.k
        ty = self.load_ty(s)
        nb = NBYTES.get(ty, 4)
        shared = s.input in self.smem
        flat = self.flat(s.index, self.shape_of(s.input))
        for i, name in enumerate(s.names):
            f = self._iadd(flat, str(i)) if i else flat
            addr = self.saddr(s.input, f) if shared else self.gaddr(s.input, f, nb)
            space = "shared" if shared else "global"
            if ty in WIDEN:
                h = k.reg("h")
                k(f"ld.{space}.b16 {h}, [{addr}];")
                r = k.reg("f")
                k(f"cvt.f32.{ty} {r}, {h};")
                self.vals[name] = (r, "f32")
            else:
                cty = _calc_ty(ty)
                r = k.reg(REG.get(cty, "r"))
                lt = LDTY.get(ty, "f32")
                if lt in ("u8", "s8", "u16", "s16"):
                    k(f"ld.{space}.{lt} {r}, [{addr}];")
                    if ty == "bool":
                        k(f"and.b32 {r}, {r}, 1;")
                else:
                    k(f"ld.{space}.{lt} {r}, [{addr}];")
                self.vals[name] = (r, cty)

    def convert(self, v, src, dst):
        """C conversion of a computed value (reference ``convert_reg``)."""
        if src == dst:
            return v
        k = self.k
        if src in ("i32", "u32", "bool") and dst in ("i32", "u32", "bool"):
            return v
        if src in ("i64", "u64") and dst in ("i64", "u64"):
            return v
        r = k.reg(REG[dst])
        if dst in ("f32", "f64") and src in ("f32", "f64"):
            k(f"cvt{'.rn' if dst == 'f32' else ''}.{dst}.{src} {r}, {v};")
        elif dst in ("f32", "f64"):
            k(f"cvt.rn.{dst}.{PTY[src]} {r}, {v};")
        elif src in ("f32", "f64"):
            if dst == "bool":
                p = k.reg("p")
                k(f"setp.ne.{src} {p}, {v}, {f32_hex(0) if src == 'f32' else f64_hex(0)};")
                k(f"selp.u32 {r}, 1, 0, {p};")
            else:
                k(f"cvt.rzi.{PTY[dst]}.{src} {r}, {v};")
        else:
            k(f"cvt.{PTY[dst]}.{PTY[src]} {r}, {v};")
        return r

    def s_Assign(self, s):
        if s.dtype is not None:
            ty = _calc_ty(s.dtype.name)
        else:
            ty = self.vals[s.args[0]][1]
        op = s.op.name
        args = [self.vals[a] for a in s.args]
        self.vals[s.name] = self.op(op, ty, args)

    def s_Let(self, s):
        k = self.k
        ty = s.dtype.name if s.dtype is not None else "f32"
        t = kind(s.value)
        if ty in INT_TYPES:
            self.ints[s.name] = self.ival(s.value)
            return
        if t == "Literal":
            cty = _calc_ty(ty)
            r = k.reg(REG[cty])
            lit = f32_hex(float(s.value.value)) if cty == "f32" else f64_hex(float(s.value.value))
            k(f"mov.{cty} {r}, {lit};")
            self.vals[s.name] = (r, cty)
        elif t == "Var" and s.value.name in self.vals:
            # an SSA binding: a copy, so that an in-place update of the source
            # (an Accum of it, later or in a later loop iteration) leaves this
            # name's value alone; ptxas drops the copy where nothing updates it
            src, cty = self.vals[s.value.name]
            if isinstance(src, str) and src.startswith("%"):
                r = k.reg(REG[cty])
                k(f"mov.{MOVTY[REG[cty]]} {r}, {src};")
                src = r
            self.vals[s.name] = (src, cty)
        elif t == "FlatIndex":
            self.ints[s.name] = self.ival(s.value)
        else:
            raise NotImplementedError(f"Let value {t}")

    def s_Init(self, s):
        k = self.k
        ty = _calc_ty(s.dtype.name)
        r = k.reg(REG[ty])
        if ty in ("f32", "f64"):
            lit = f32_hex(float(s.identity)) if ty == "f32" else f64_hex(float(s.identity))
            k(f"mov.{ty} {r}, {lit};")
        else:
            k(f"mov.{PTY[ty]} {r}, {int(s.identity)};")
        self.vals[s.name] = (r, ty)

    def accum_reg(self, s):
        if s.name in self.vals:
            return self.vals[s.name]
        k = self.k
        ty = _calc_ty(s.dtype.name if s.dtype is not None else "f32")
        r = k.reg(REG[ty])
        k(f"mov.{PTY[ty] if ty not in ('f32', 'f64') else ty} {r}, {self._identity(s.op.name, ty)};")
        self.vals[s.name] = (r, ty)
        return r, ty

    @staticmethod
    def _identity(op, ty):
        if ty == "f32":
            return f32_hex(identity_f32(op))
        if ty == "f64":
            return f64_hex(identity_f32(op))
        big = 9223372036854775807 if ty in ("i64", "u64") else 2147483647
        return {"add": "0", "multiply": "1", "maximum": str(-big - 1), "minimum": str(big)}[op]

    def s_Accum(self, s):
        reg, ty = self.accum_reg(s)
        left = self.vals[s.base] if s.base else (reg, ty)
        r, _ = self.op(s.op.name, ty, [left, self.vals[s.value]])
        self.k(f"mov.{'b32' if REG[ty] in ('f', 'r') else 'b64'} {reg}, {r};")
        self.vals[s.name] = (reg, ty)

    def s_Write(self, s):
        k = self.k
        ty = s.value_dtype.name
        nb = NBYTES.get(ty, 4)
        if getattr(s, "swizzle", None) not in (None, "NONE"):
            raise NotImplementedError(f"Write swizzle {s.swizzle!r}")
        shared = s.output in self.smem
        if shared:
            ty = self.smem[s.output]["ty"]
            nb = self.smem[s.output]["nbytes"]
        flat = self.flat(s.index, self.shape_of(s.output))
        for i, vname in enumerate(s.values):
            v, vty = self.vals[vname]
            f = self._iadd(flat, str(i)) if i else flat
            addr = self.saddr(s.output, f) if shared else self.gaddr(s.output, f, nb)
            space = "shared" if shared else "global"
            if ty in WIDEN:
                fv = self.convert(v, vty, "f32")
                h = k.reg("h")
                k(f"cvt.rn.{ty}.f32 {h}, {fv};")
                if s.atomic:
                    k(f"red.{space}.add.noftz.{ty} [{addr}], {h};")
                else:
                    k(f"st.{space}.b16 [{addr}], {h};")
                continue
            cty = _calc_ty(ty)
            cv = self.convert(v, vty, cty)
            st = LDTY.get(ty, "f32").replace("s8", "u8").replace("s16", "u16")
            if s.atomic:
                at = {"f32": "f32", "f64": "f64", "i32": "s32", "u32": "u32", "i64": "u64",
                      "u64": "u64"}.get(ty)
                if at is None:
                    raise NotImplementedError(f"atomic add of {ty}")
                k(f"red.{space}.add.{at} [{addr}], {cv};")
            else:
                if st in ("u8", "u16") and REG.get(cty) == "rd":
                    t = k.reg("r")
                    k(f"cvt.u32.u64 {t}, {cv};")
                    cv = t
                k(f"st.{space}.{st} [{addr}], {cv};")

    def s_Cond(self, s):
        k = self.k
        p = self.pred(s.cond)
        els = k.label("ELSE")
        k(f"@!{p} bra {els};")
        saved = dict(self.ints)
        self.body(s.body)
        self.ints = saved
        if s.else_body:
            end = k.label("ENDIF")
            k(f"bra {end};")
            k.mark(els)
            self.body(s.else_body)
            self.ints = dict(saved)
            k.mark(end)
        else:
            k.mark(els)

    def init_accumulators(self, body):
        for s in body:
            t = kind(s)
            if t == "Accum":
                self.accum_reg(s)
            elif t == "Cond":
                for sub in (s.body, s.else_body):
                    if sub:
                        self.init_accumulators(sub)

    UNROLL_CAP = 128

    # ---------------------------------------------------------- carried state
    # TASK.md's Carry / Pre (defined by the IR vocabulary, lowered by no
    # reference code): a carried-state cell is named by its carrier and a
    # literal index; its loop is the innermost loop around the Carry, whose
    # iterations are the steps.  Each step starts with next = state (cells
    # no Carry of the step sets keep their values), Carry sets next, Pre
    # reads state (the previous step's value, the seed on the first step),
    # and the step ends with state = next; after the loop Pre reads the final
    # value.
    def _cell_key(self, carrier, index):
        key = []
        for e in index or ():
            v = self.ival(e)
            if not _is_imm(v):
                raise NotImplementedError("carried-state cell with a run-time index")
            key.append(int(v))
        return (carrier, tuple(key))

    def _carries(self, body):
        """Carry statements of this loop's steps (not of nested loops)."""
        out = []
        for st in body:
            kd = kind(st)
            if kd == "Carry":
                out.append(st)
            elif kd == "Cond":
                out += self._carries(st.body) + self._carries(st.else_body or ())
        return out

    def _open_cells(self, body):
        """Create (state = seed) the cells this loop carries; return them."""
        k = self.k
        cells = []
        for st in self._carries(body):
            key = self._cell_key(st.name, st.index)
            if key not in self.cells:
                ty = _calc_ty(st.dtype.name if st.dtype is not None else "f32")
                state, nxt = k.reg(REG[ty]), k.reg(REG[ty])
                lit = float(st.seed) if ty in ("f32", "f64") else int(st.seed)
                if ty == "f32":
                    k(f"mov.f32 {state}, {f32_hex(lit)};")
                elif ty == "f64":
                    k(f"mov.f64 {state}, {f64_hex(lit)};")
                else:
                    k(f"mov.{PTY[ty]} {state}, {lit};")
                self.cells[key] = [state, nxt, ty]
            if key not in cells:
                cells.append(key)
        return cells

    def _step(self, cells, begin: bool):
        for key in cells:
            state, nxt, ty = self.cells[key]
            mv = MOVTY[REG[ty]]
            if begin:
                self.k(f"mov.{mv} {nxt}, {state};")
            else:
                self.k(f"mov.{mv} {state}, {nxt};")

    def s_Carry(self, s):
        key = self._cell_key(s.name, s.index)
        if key not in self.cells:        # a Carry outside any loop: one step
            self._open_cells((s,))
            self._step([key], True)
        _, nxt, ty = self.cells[key]
        v, vty = self.vals[s.value] if isinstance(s.value, str) else \
            (f32_hex(float(s.value.value)), "f32")
        v = self.convert(v, vty, ty)
        self.k(f"mov.{MOVTY[REG[ty]]} {nxt}, {v};")

    def s_Pre(self, s):
        key = self._cell_key(s.carrier, s.index)
        if key not in self.cells:
            raise NotImplementedError(f"Pre of {s.carrier} before any Carry of it")
        state, _, ty = self.cells[key]
        r = self.k.reg(REG[ty])
        self.k(f"mov.{MOVTY[REG[ty]]} {r}, {state};")
        self.vals[s.name] = (r, ty)

    def s_Select(self, s):
        """``name`` = the value of the branch whose coordinate predicate holds
        (TASK.md ``Select``: branches of (value, select)); evaluated as a
        chain of selects from the last branch back, so the first branch
        whose predicate holds wins."""
        k = self.k
        branches = [(b.value, b.select) if hasattr(b, "select") else (b[0], b[1])
                    for b in s.branches]
        if not branches:
            raise NotImplementedError("Select without branches")
        vals = []
        for v, _ in branches:
            if isinstance(v, str):
                vals.append(self.vals[v])
            else:
                vals.append((self.fval(v, "f32"), "f32"))
        ty = vals[0][1]
        r = k.reg(REG[ty])
        k(f"mov.{MOVTY[REG[ty]]} {r}, {self.convert(vals[-1][0], vals[-1][1], ty)};")
        for (v, vty), (_, sel) in list(zip(vals, branches))[-2::-1]:
            p = self.pred(sel)
            k(f"selp.{'b32' if REG[ty] in ('f', 'r') else 'b64'} {r}, "
              f"{self.convert(v, vty, ty)}, {r}, {p};")
        self.vals[s.name] = (r, ty)

    def s_ZeroPrologue(self, s):
        """Zero ``words`` 32-bit words of buffer ``dst`` (another kernel's
        atomic accumulator), every thread of the grid a strided share, in
        place of a memset before that kernel (TASK.md ``ZeroPrologue``)."""
        k = self.k
        words = int(s.words.value if hasattr(s.words, "value") else s.words)
        total = self.ctx.total_threads
        i = k.reg("rd")
        k(f"mov.u64 {i}, {self.gid64};")
        top, out = k.label("ZERO"), k.label("ZERO_END")
        k.mark(top)
        p = k.reg("p")
        k(f"setp.ge.u64 {p}, {i}, {words};")
        k(f"@{p} bra {out};")
        a = k.reg("rd")
        k(f"shl.b64 {a}, {i}, 2;")
        k(f"add.s64 {a}, {a}, {self.base[s.dst]};")
        k(f"st.global.b32 [{a}], 0;")
        k(f"add.s64 {i}, {i}, {total};")
        k(f"bra {top};")
        k.mark(out)

    def _loop(self, axis, start, step, end, body, seed):
        k = self.k
        if seed:
            self.init_accumulators(body)
        cells = self._open_cells(body)
        if cells:
            body = (_StepMark(cells, True),) + tuple(body) + (_StepMark(cells, False),)
        name = axis.name
        saved = self.ints.get(name)
        if _is_imm(start) and _is_imm(step) and _is_imm(end) and int(step) > 0:
            trip = max(0, -(-(int(end) - int(start)) // int(step)))
            if 1 < trip <= self.UNROLL_CAP and not any(
                    kind(x) in ("Loop", "StridedLoop") for x in walk(body)):
                # one copy of the body per iteration, the axis a constant.
                # Each copy starts from the bindings the loop form's body
                # sees on every iteration (those made before the loop), so
                # what the loop form re-executes per iteration (lazily
                # initialised accumulators, rebindings) is re-executed by
                # every copy; accumulators keep their registers, so their
                # state carries from copy to copy as from iteration to
                # iteration, and after the loop the last copy's bindings hold
                before_v, before_i = dict(self.vals), dict(self.ints)
                for it in range(trip):
                    self.vals = dict(before_v)
                    self.ints = dict(before_i)
                    self.ints[name] = str(int(start) + it * int(step))
                    self.body(body)
                if saved is None:
                    self.ints.pop(name, None)
                else:
                    self.ints[name] = saved
                return
        v = k.reg("r")
        k(f"mov.u32 {v}, {start};")
        top, out = k.label("LOOP"), k.label("ENDLOOP")
        k.mark(top)
        p = k.reg("p")
        k(f"setp.ge.s32 {p}, {v}, {end};")
        k(f"@{p} bra {out};")
        self.ints[name] = v
        self.body(body)
        k(f"add.s32 {v}, {v}, {step};")
        k(f"bra {top};")
        k.mark(out)
        if saved is None:
            self.ints.pop(name, None)
        else:
            self.ints[name] = saved

    def s_Loop(self, s):
        self._loop(s.axis, "0", "1", str(dim(s.axis.extent)), s.body, s.seed)

    def s_StridedLoop(self, s):
        start = self.ival(s.start)
        step = self.ival(s.step)
        end = self.ival(s.end) if s.end is not None else str(dim(s.axis.extent))
        if _is_imm(end):
            pass
        self._loop(s.axis, start, step, end, s.body, s.seed)

    def s_Smem(self, s):
        extents = tuple(int(e) for e in s.extents)
        ty = SMEM_TY.get(s.dtype, s.dtype if s.dtype in NBYTES else "f32")
        nb = NBYTES.get(ty, 4)
        size = prod(extents) * nb
        align = max(int(s.align or 0), (4 if nb <= 4 else 2) * nb, 4)
        info = {"extents": extents, "ty": ty, "nbytes": nb, "align": align}
        if self.dynamic:
            off = -(-self.smem_used // align) * align
            self.smem_used = off + size
            self.max_align = max(self.max_align, align)
            info["off"] = off
        else:
            sym = f"__emmy_s_{s.name}"
            self.k.decl(f".shared .align {align} .b8 {sym}[{max(size, 1)}];")
            info["sym"] = sym
        self.smem[s.name] = info

    def s_Sync(self, s):
        bid = int(s.barrier_id or 0)
        if self._wg is not None and not s.warp:
            # threads' shared-memory writes become visible to the tensor
            # core's async proxy before the barrier orders them
            self.k("fence.proxy.async.shared::cta;")
        if s.warp:
            self.k("bar.warp.sync 0xffffffff;")
        elif bid:
            if s.count is None:
                raise NotImplementedError("named barrier requires a thread count")
            self.k(f"bar.sync {bid}, {s.count};")
        else:
            self.k("bar.sync 0;")

    def s_WarpShuffle(self, s):
        k = self.k
        off = s.length // 2
        while off > 0:
            mask = k.reg("r")
            k(f"activemask.b32 {mask};")
            for st, sb in zip(s.state, s.state_b):
                v, ty = self.vals[st]
                if REG[ty] in ("fd", "rd"):
                    lo, hi = k.reg("r"), k.reg("r")
                    k(f"mov.b64 {{{lo}, {hi}}}, {v};")
                    k(f"shfl.sync.bfly.b32 {lo}, {lo}, {off}, 0x1f, {mask};")
                    k(f"shfl.sync.bfly.b32 {hi}, {hi}, {off}, 0x1f, {mask};")
                    peer = k.reg(REG[ty])
                    k(f"mov.b64 {peer}, {{{lo}, {hi}}};")
                else:
                    b = k.reg("r")
                    k(f"mov.b32 {b}, {v};")
                    k(f"shfl.sync.bfly.b32 {b}, {b}, {off}, 0x1f, {mask};")
                    peer = k.reg(REG[ty])
                    k(f"mov.b32 {peer}, {b};")
                self.vals[sb] = (peer, ty)
            self.body(s.combine_states)
            off //= 2

    def s_TreeHalve(self, s):
        k = self.k
        tid = self.ival(I_Var(s.tid_var))
        scale, root = 1, "0"
        if s.inner is not None:
            iv, scale = s.inner
            root = self.ival(I_Var(iv))
        base = self._iadd(self._imul(tid, scale), root)
        bid = int(s.barrier_id or 0)
        # a tree indexed by the warp (the reference's form, compile.py:1814-1857)
        # runs every step in all 32 lanes of a warp on the same entries: the
        # lanes' loads must all complete before any store (independent thread
        # scheduling lets one lane run ahead) and one lane stores
        warp_tree = s.inner is None and tid == getattr(self, "builtin_warp", None)
        # the tree reads entries [0, length) (times ``scale``, plus the inner
        # root < scale): a tree longer than its buffer would read shared
        # memory outside it, so such an IR is refused rather than lowered
        for buf in s.bufs:
            entries = prod(self.smem[buf]["extents"])
            if (s.length - 1) * scale + (scale - 1) >= entries:
                raise NotImplementedError(
                    f"TreeHalve of length {s.length} (scale {scale}) reads past its "
                    f"shared buffer {buf} of {entries} entries")
        # halving steps (n live entries -> ceil(n/2)); for a power of two this
        # is the plain tree: level = n/2, entries [0, level) fold [level, n)
        steps = []
        n = s.length
        while n > 1:
            h = (n + 1) // 2
            steps.append((n - h, h))      # (active entries, distance)
            n = h
        for active, level in steps:
            p = k.reg("p")
            t = tid
            if _is_imm(t):
                t2 = k.reg("r")
                k(f"mov.u32 {t2}, {t};")
                t = t2
            k(f"setp.lt.s32 {p}, {t}, {active};")
            skip = k.label("TREE_SKIP")
            k(f"@!{p} bra {skip};")
            other = self._iadd(base, str(level * scale))
            for buf, st, sb in zip(s.bufs, s.state, s.state_b):
                ty = _calc_ty(self.smem[buf]["ty"])
                a = k.reg(REG[ty])
                k(f"ld.shared.{ty if ty in ('f32', 'f64') else PTY[ty]} {a}, [{self.saddr(buf, base)}];")
                b = k.reg(REG[ty])
                k(f"ld.shared.{ty if ty in ('f32', 'f64') else PTY[ty]} {b}, [{self.saddr(buf, other)}];")
                self.vals[st] = (a, ty)
                self.vals[sb] = (b, ty)
            self.body(s.combine_states)
            lead = ""
            if warp_tree:
                am = k.reg("r")
                k(f"activemask.b32 {am};")
                k(f"bar.warp.sync {am};")
                pl = k.reg("p")
                k(f"setp.eq.u32 {pl}, {self.ints['lane']}, 0;")
                lead = f"@{pl} "
            for buf, st in zip(s.bufs, s.state):
                ty = _calc_ty(self.smem[buf]["ty"])
                v = self.convert(*self.vals[st], ty)
                k(f"{lead}st.shared.{ty if ty in ('f32', 'f64') else PTY[ty]} "
                  f"[{self.saddr(buf, base)}], {v};")
            k.mark(skip)
            if bid and s.barrier_count is not None:
                k(f"bar.sync {bid}, {s.barrier_count};")
            else:
                k("bar.sync 0;")
        for buf, st in zip(s.bufs, s.state):
            ty = _calc_ty(self.smem[buf]["ty"])
            r = k.reg(REG[ty])
            k(f"ld.shared.{ty if ty in ('f32', 'f64') else PTY[ty]} {r}, [{self.saddr(buf, root)}];")
            self.vals[st] = (r, ty)

    def s_CpAsyncCopy(self, s):
        k = self.k
        info = self.smem[s.smem]
        flat = self.flat(s.smem_index, info["extents"])
        if s.lane_index is not None:
            cols = info["extents"][-1]
            lf = self._iadd(self._imul(self.ival(s.lane_index[0]), cols),
                            self.ival(s.lane_index[1]))
            flat = self._iadd(flat, lf)
        flat = self.apply_swizzle(flat, s.swizzle)
        sa = self.saddr(s.smem, flat)
        src_ty = self.ctx.bufs.dtypes.get(s.src, "f32")
        ga = self.gaddr(s.src, self.flat(s.src_index, self.shape_of(s.src)), NBYTES.get(src_ty, 4))
        ins = "cp.async.cg.shared.global" if s.nbytes == 16 else "cp.async.ca.shared.global"
        k(f"{ins} [{sa}], [{ga}], {s.nbytes};")

    def apply_swizzle(self, flat, swizzle):
        """A shared-memory flat element index under the vocabulary's swizzle
        (the reference's ``apply_swizzle``, ``compile.py:1706-1730``):
        ``"B128"`` / ``"B64"`` / ``"B32"`` with an optional ``@shift`` (default
        6) XOR 8-element chunks by (index >> shift) & 7 / 3 / 1."""
        if swizzle in (None, "NONE"):
            return flat
        k = self.k
        sw = str(swizzle)
        mode, shift = (sw.split("@") + ["6"])[:2] if "@" in sw else (sw, "6")
        mask = {"B128": 7, "B64": 3, "B32": 1}.get(mode)
        if mask is None:
            raise NotImplementedError(f"swizzle {swizzle!r}")
        if _is_imm(flat):
            e = int(flat)
            return str(e ^ (((e >> int(shift)) & mask) << 3))
        t1 = k.reg("r")
        k(f"shr.u32 {t1}, {flat}, {shift};")
        k(f"and.b32 {t1}, {t1}, {mask};")
        k(f"shl.b32 {t1}, {t1}, 3;")
        t2 = k.reg("r")
        k(f"xor.b32 {t2}, {flat}, {t1};")
        return t2

    # ------------------------------------------------- TMA and mbarriers
    # The reference defines these nodes without lowering them (TASK.md
    # "Transport into shared memory", starred).  A TmaDescriptor becomes a
    # trailing 128-byte tensor-map parameter plus an ``// @emmy tmap`` line
    # the host harness encodes; TmaLoad is one ``cp.async.bulk.tensor`` by each
    # thread that reaches it; mbarrier waits are bounded by %globaltimer.
    TMA_DTYPE = {"u8": 0, "u16": 1, "u32": 2, "i32": 3, "u64": 4, "i64": 5, "f16": 6,
                 "f32": 7, "f64": 8, "bf16": 9}
    TMA_SWIZZLE = {None: 0, "NONE": 0, "B32": 1, "B64": 2, "B128": 3}
    # destination alignment a box copy needs in shared memory, by swizzle
    TMA_SMEM_ALIGN = {0: 128, 1: 256, 2: 512, 3: 1024}
    WAIT_NS = 2_000_000_000

    def _declare_mbarriers(self, tile):
        """mbarriers the IR uses without declaring an Smem array for them get
        one static 8-byte slot per literal slot index."""
        declared = {s.name for s in walk(tile.body) if kind(s) == "Smem"}
        need = {}
        for s in walk(tile.body):
            kd = kind(s)
            if kd in ("MbarrierInit", "MbarrierArriveExpectTx", "MbarrierArrive", "MbarrierWait",
                      "TmaLoad"):
                name = s.mbar
                slot = s.mbar_slot if kd == "TmaLoad" else s.slot
                if name in declared:
                    continue
                v = self._literal_int(slot)
                if v is None:
                    raise NotImplementedError(
                        f"mbarrier {name} indexed by an expression needs an Smem declaration")
                need[name] = max(need.get(name, 0), v + 1)
        for name, n in need.items():
            sym = f"__emmy_mbar_{name}"
            self.k.decl(f".shared .align 8 .b8 {sym}[{8 * n}];")
            self.smem[name] = {"extents": (n,), "ty": "u64", "nbytes": 8, "sym": sym,
                               "static": True}

    @staticmethod
    def _literal_int(e):
        if e is None:
            return 0
        if isinstance(e, int):
            return e
        if kind(e) == "Literal":
            return int(e.value)
        return None

    def _slot(self, e) -> str:
        if e is None:
            return "0"
        if isinstance(e, int):
            return str(e)
        return self.ival(e)

    def mbar_addr(self, name, slot) -> str:
        if name not in self.smem:
            raise NotImplementedError(f"mbarrier {name} is not declared")
        info = self.smem[name]
        if info.get("static"):
            k = self.k
            base = k.reg("r")
            k(f"mov.u32 {base}, {info['sym']};")
            sl = self._slot(slot)
            if _is_imm(sl):
                if int(sl):
                    k(f"add.u32 {base}, {base}, {8 * int(sl)};")
                return base
            a = k.reg("r")
            k(f"mad.lo.s32 {a}, {sl}, 8, {base};")
            return a
        return self.saddr(name, self._slot(slot))

    def _status(self):
        if not getattr(self, "_has_status", False):
            self.k.decl(".global .align 4 .u32 __emmy_status;")
            self._has_status = True
        r = self.k.reg("rd")
        self.k(f"mov.u64 {r}, __emmy_status;")
        return r

    def s_TmaDescriptor(self, s):
        k = self.k
        ty = getattr(s.dtype, "name", s.dtype) or self.ctx.bufs.dtypes.get(s.src_buf, "f32")
        if ty not in self.TMA_DTYPE:
            raise NotImplementedError(f"TMA dtype {ty}")
        shape = [dim(d) for d in s.src_shape]
        box = [dim(d) for d in s.box_extents]
        if len(shape) != len(box) or not 1 <= len(shape) <= 5:
            raise NotImplementedError("TMA descriptor rank")
        if s.src_buf not in self.base:
            raise NotImplementedError(f"TMA source {s.src_buf} is not a kernel argument")
        if prod(shape) > self.ctx.bufs.size(s.src_buf):
            raise NotImplementedError(f"TMA shape {shape} exceeds buffer {s.src_buf}")
        nb = NBYTES[ty]
        sw = self.TMA_SWIZZLE.get(s.swizzle if s.swizzle is None else str(s.swizzle))
        if sw is None:
            raise NotImplementedError(f"TMA swizzle {s.swizzle}")
        dims = list(reversed(shape))
        boxr = list(reversed(box))
        strides, acc = [], nb
        for d in dims[:-1]:
            acc *= d
            strides.append(acc)
        param = f"tmap_{s.name}"
        k.params.append((param, ".align 64 .b8", "[128]"))
        sdir = f" strides={','.join(map(str, strides))}" if strides else ""
        k.directive(f"tmap {param} buf={s.src_buf} dtype={self.TMA_DTYPE[ty]} "
                    f"dims={','.join(map(str, dims))}{sdir} box={','.join(map(str, boxr))} "
                    f"swizzle={sw}")
        r = k.reg("rd")
        k(f"mov.u64 {r}, param_{param};")
        k(f"cvta.param.u64 {r}, {r};")
        self.tmaps[s.name] = (r, {"ty": ty, "nb": nb, "box": box, "swizzle": sw,
                                  "bytes": prod(box) * nb})

    def s_TmaLoad(self, s):
        k = self.k
        if s.desc not in self.tmaps:
            raise NotImplementedError(f"TmaLoad of undeclared descriptor {s.desc}")
        tm, info = self.tmaps[s.desc]
        coords = [self.ival(c) for c in s.coords]
        if len(coords) != len(info["box"]):
            raise NotImplementedError("TmaLoad coordinate count")
        coords = list(reversed(coords))        # innermost first
        per16 = 16 // info["nb"] if info["nb"] < 16 else 1
        sinfo = self.smem[s.smem]
        align = self.TMA_SMEM_ALIGN[info["swizzle"]]
        if not self.dynamic and int(sinfo.get("align", 0) or 0) < align:
            raise NotImplementedError(f"TMA destination {s.smem} must be {align}-byte aligned")
        dst = self.saddr(s.smem, self.flat(s.smem_index, sinfo["extents"]))
        mb = self.mbar_addr(s.mbar, s.mbar_slot)
        skip = k.label("TMA_SKIP")
        done = k.label("TMA_DONE")
        # the innermost coordinate times the element size must be a multiple
        # of 16 bytes, and the destination aligned for the swizzle mode; a copy
        # that breaks either is not issued (status 9) -- waits on its barrier
        # then time out instead of the copy faulting
        if _is_imm(coords[0]):
            if int(coords[0]) % per16:
                raise NotImplementedError("TMA innermost coordinate not 16-byte aligned")
        else:
            t = k.reg("r")
            k(f"and.b32 {t}, {coords[0]}, {per16 - 1};")
            p = k.reg("p")
            k(f"setp.ne.u32 {p}, {t}, 0;")
            k(f"@{p} bra {skip};")
        t2 = k.reg("r")
        k(f"and.b32 {t2}, {dst}, {align - 1};")
        p2 = k.reg("p")
        k(f"setp.ne.u32 {p2}, {t2}, 0;")
        k(f"@{p2} bra {skip};")
        cs = []
        for c in coords:
            if _is_imm(c):
                r = k.reg("r")
                k(f"mov.u32 {r}, {int(c)};")
                c = r
            cs.append(c)
        n = len(cs)
        k(f"cp.async.bulk.tensor.{n}d.shared::cluster.global.mbarrier::complete_tx::bytes "
          f"[{dst}], [{tm}, {{{', '.join(cs)}}}], [{mb}];")
        k(f"bra {done};")
        k.mark(skip)
        st = self._status()
        k(f"st.global.u32 [{st}], 9;")
        k.mark(done)

    def s_MbarrierInit(self, s):
        a = self.mbar_addr(s.mbar, s.slot)
        cnt = self.ival(s.count) if not isinstance(s.count, int) else str(s.count)
        self.k(f"mbarrier.init.shared::cta.b64 [{a}], {cnt};")
        self.k("fence.mbarrier_init.release.cluster;")

    def s_MbarrierArriveExpectTx(self, s):
        a = self.mbar_addr(s.mbar, s.slot)
        nb = self.ival(s.bytes_) if not isinstance(s.bytes_, int) else str(s.bytes_)
        self.k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{a}], {nb};")

    def s_MbarrierArrive(self, s):
        a = self.mbar_addr(s.mbar, s.slot)
        self.k(f"mbarrier.arrive.shared::cta.b64 _, [{a}];")

    def s_MbarrierWait(self, s):
        k = self.k
        a = self.mbar_addr(s.mbar, s.slot)
        ph = self.ival(s.phase) if not isinstance(s.phase, int) else str(s.phase)
        par = k.reg("r")
        if _is_imm(ph):
            k(f"mov.u32 {par}, {int(ph) & 1};")
        else:
            k(f"and.b32 {par}, {ph}, 1;")
        self.bounded_parity_wait(a, par)

    def bounded_parity_wait(self, a, par):
        """Wait until the mbarrier at shared address ``a`` completes the phase
        of parity ``par``, for at most ``WAIT_NS`` of %globaltimer; on expiry
        record status 8 in ``__emmy_status`` and go on."""
        k = self.k
        p = k.reg("p")
        top, ok = k.label("MBAR_WAIT"), k.label("MBAR_OK")
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{a}], {par};")
        k(f"@{p} bra {ok};")
        t0 = k.reg("rd")
        k(f"mov.u64 {t0}, %globaltimer;")
        k.mark(top)
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{a}], {par};")
        k(f"@{p} bra {ok};")
        t1 = k.reg("rd")
        k(f"mov.u64 {t1}, %globaltimer;")
        k(f"sub.s64 {t1}, {t1}, {t0};")
        q = k.reg("p")
        k(f"setp.lt.s64 {q}, {t1}, {self.WAIT_NS};")
        k(f"@{q} bra {top};")
        st = self._status()
        k(f"st.global.u32 [{st}], 8;")
        k.mark(ok)

    def s_SetMaxNReg(self, s):
        # honoured as the hint it is: register use stays ptxas's choice.  An
        # .inc is only safe when the launch's registers cover every
        # warpgroup's share, which this lowering cannot see, and an .inc that
        # asks for more than was freed waits forever
        self.k.comment(f"SetMaxNReg {s.direction} {s.count}: hint, not emitted")

    def s_CpAsyncCommit(self, s):
        self.k("cp.async.commit_group;")

    def s_CpAsyncWait(self, s):
        self.k(f"cp.async.wait_group {int(s.group)};")

    # --------------------------------------------------------- elementwise ops
    def op(self, op, ty, args):
        """Emit ``op(args)`` computed in ``ty``; returns (register, type)."""
        k = self.k
        if op in CMP:
            src = args[0][1]
            cty = "f64" if any(a[1] == "f64" for a in args) else \
                "f32" if any(a[1] == "f32" for a in args) else src
            a = [self.convert(v, t, cty) for v, t in args]
            p = k.reg("p")
            pt = cty if cty in ("f32", "f64") else PTY[cty]
            # C '!=' is true when either side is NaN: the unordered form for
            # floats (reference compile.py:1532-1551 negates an ordered eq)
            cmp = "neu" if op == "not_equal" and cty in ("f32", "f64") else CMP[op]
            k(f"setp.{cmp}.{pt} {p}, {a[0]}, {a[1]};")
            r = k.reg("r")
            k(f"selp.u32 {r}, 1, 0, {p};")
            res = (r, "bool")
            return (self.convert(r, "bool", ty), ty) if ty != "bool" else res
        if op == "where":
            cv, ct = args[0]
            p = k.reg("p")
            if ct in ("f32", "f64"):
                k(f"setp.ne.{ct} {p}, {cv}, {f32_hex(0) if ct == 'f32' else f64_hex(0)};")
            else:
                k(f"setp.ne.{'s64' if REG[ct] == 'rd' else 's32'} {p}, {cv}, 0;")
            a = self.convert(*args[1], ty)
            b = self.convert(*args[2], ty)
            r = k.reg(REG[ty])
            k(f"selp.{PTY[ty] if ty not in ('f32', 'f64') else ty} {r}, {a}, {b}, {p};")
            return r, ty
        if op in ("logical_and", "logical_or", "logical_xor", "logical_not"):
            a = [self.convert(v, t, "bool") for v, t in args]
            r = k.reg("r")
            if op == "logical_not":
                k(f"xor.b32 {r}, {a[0]}, 1;")
            else:
                k(f"{op.split('_')[1]}.b32 {r}, {a[0]}, {a[1]};")
            return r, "bool"
        a = [self.convert(v, t, ty) for v, t in args]
        if ty == "f32":
            return self._op_f32(op, a), "f32"
        if ty == "f64":
            return self._op_f64(op, a), "f64"
        if ty in ("i32", "u32", "i64", "u64", "bool"):
            return self._op_int(op, ty, a), ty
        raise NotImplementedError(f"op {op} on {ty}")

    def _op_f32(self, op, a):
        k = self.k
        try:
            return emit_op_f32(k, op, a)
        except UnsupportedOp:
            pass
        d = k.reg("f")
        if op == "pow":
            return self._pow_f32(a[0], a[1])
        if op in ("sin", "cos"):
            return self._sincos(op, a[0])
        if op == "erf":
            return self._erf(a[0])
        if op in ("fmod", "mod", "remainder", "floor_divide"):
            q = k.reg("f")
            k(f"div.rn.f32 {q}, {a[0]}, {a[1]};")
            t = k.reg("f")
            # floor_divide floors; mod / remainder / fmod are C '%' on floats
            # (truncated quotient, the result keeps the dividend's sign), as
            # the reference lowers all three (compile.py:752-770)
            rnd = "rmi" if op == "floor_divide" else "rzi"
            k(f"cvt.{rnd}.f32.f32 {t}, {q};")
            if op == "floor_divide":
                return t
            m = k.reg("f")
            k(f"mul.rn.f32 {m}, {t}, {a[1]};")
            k(f"sub.rn.f32 {d}, {a[0]}, {m};")
            return d
        if op == "sign":
            p, n = k.reg("p"), k.reg("p")
            k(f"setp.gt.f32 {p}, {a[0]}, 0f00000000;")
            k(f"setp.lt.f32 {n}, {a[0]}, 0f00000000;")
            k(f"selp.f32 {d}, 0f3F800000, 0f00000000, {p};")
            k(f"@{n} mov.f32 {d}, 0fBF800000;")
            return d
        if op == "softplus":
            # log(1 + e^-|x|) + max(x, 0)
            ab = k.reg("f")
            k(f"abs.f32 {ab}, {a[0]};")
            k(f"neg.f32 {ab}, {ab};")
            e = emit_exp(k, ab)
            s = k.reg("f")
            k(f"add.rn.f32 {s}, {e}, 0f3F800000;")
            l2 = k.reg("f")
            k(f"lg2.approx.f32 {l2}, {s};")
            k(f"mul.rn.f32 {l2}, {l2}, {f32_hex(LN2)};")
            mx = k.reg("f")
            k(f"max.f32 {mx}, {a[0]}, 0f00000000;")
            k(f"add.rn.f32 {d}, {l2}, {mx};")
            return d
        if op == "log1p":
            s = k.reg("f")
            k(f"add.rn.f32 {s}, {a[0]}, 0f3F800000;")
            k(f"lg2.approx.f32 {d}, {s};")
            k(f"mul.rn.f32 {d}, {d}, {f32_hex(LN2)};")
            return d
        if op == "frac":
            t = k.reg("f")
            k(f"cvt.rzi.f32.f32 {t}, {a[0]};")
            k(f"sub.rn.f32 {d}, {a[0]}, {t};")
            return d
        raise NotImplementedError(f"op {op} (f32)")

    def _pow_f32(self, x, y):
        """x^y = 2^(y log2|x|); a negative base needs an integral exponent
        (odd exponents keep the sign), and x^0 = 1 for every x."""
        k = self.k
        ax = k.reg("f")
        k(f"abs.f32 {ax}, {x};")
        l2 = k.reg("f")
        k(f"lg2.approx.f32 {l2}, {ax};")
        t = k.reg("f")
        k(f"mul.rn.f32 {t}, {l2}, {y};")
        r = k.reg("f")
        k(f"ex2.approx.f32 {r}, {t};")
        yi = k.reg("f")
        k(f"cvt.rzi.f32.f32 {yi}, {y};")
        neg = k.reg("p")
        k(f"setp.lt.f32 {neg}, {x}, 0f00000000;")
        isint = k.reg("p")
        k(f"setp.eq.f32 {isint}, {yi}, {y};")
        half = k.reg("f")
        k(f"mul.rn.f32 {half}, {y}, 0f3F000000;")
        hf = k.reg("f")
        k(f"cvt.rzi.f32.f32 {hf}, {half};")
        odd = k.reg("p")
        k(f"setp.ne.f32 {odd}, {hf}, {half};")
        po = k.reg("p")
        k(f"and.pred {po}, {neg}, {odd};")
        k(f"and.pred {po}, {po}, {isint};")
        k(f"@{po} neg.f32 {r}, {r};")
        pn = k.reg("p")
        k(f"not.pred {pn}, {isint};")
        k(f"and.pred {pn}, {pn}, {neg};")
        k(f"@{pn} mov.f32 {r}, 0f7FC00000;")
        pz = k.reg("p")
        k(f"setp.eq.f32 {pz}, {y}, 0f00000000;")
        k(f"@{pz} mov.f32 {r}, 0f3F800000;")
        return r

    def _sincos(self, op, x):
        """Range-reduce in f64 (x - round(x / 2pi) * 2pi), then the hardware
        sin/cos approximation on [-pi, pi]."""
        k = self.k
        xd = k.reg("fd")
        k(f"cvt.f64.f32 {xd}, {x};")
        q = k.reg("fd")
        k(f"mul.rn.f64 {q}, {xd}, {f64_hex(1 / (2 * math.pi))};")
        k(f"cvt.rni.f64.f64 {q}, {q};")
        k(f"fma.rn.f64 {xd}, {q}, {f64_hex(-2 * math.pi)}, {xd};")
        r = k.reg("f")
        k(f"cvt.rn.f32.f64 {r}, {xd};")
        d = k.reg("f")
        k(f"{op}.approx.f32 {d}, {r};")
        return d

    def _erf(self, x):
        """Abramowitz & Stegun 7.1.26 (|error| < 1.5e-7), odd extension."""
        k = self.k
        ax = k.reg("f")
        k(f"abs.f32 {ax}, {x};")
        t = k.reg("f")
        k(f"fma.rn.f32 {t}, {ax}, {f32_hex(0.3275911)}, 0f3F800000;")
        k(f"rcp.rn.f32 {t}, {t};")
        poly = k.reg("f")
        k(f"mov.f32 {poly}, {f32_hex(1.061405429)};")
        for c in (-1.453152027, 1.421413741, -0.284496736, 0.254829592):
            k(f"fma.rn.f32 {poly}, {poly}, {t}, {f32_hex(c)};")
        k(f"mul.rn.f32 {poly}, {poly}, {t};")
        sq = k.reg("f")
        k(f"mul.rn.f32 {sq}, {ax}, {ax};")
        k(f"neg.f32 {sq}, {sq};")
        e = emit_exp(k, sq)
        y = k.reg("f")
        k(f"mul.rn.f32 {y}, {poly}, {e};")
        k(f"sub.rn.f32 {y}, 0f3F800000, {y};")
        n = k.reg("p")
        k(f"setp.lt.f32 {n}, {x}, 0f00000000;")
        k(f"@{n} neg.f32 {y}, {y};")
        return y

    def _op_f64(self, op, a):
        k = self.k
        d = k.reg("fd")
        simple = {"add": "add.rn.f64", "subtract": "sub.rn.f64", "multiply": "mul.rn.f64",
                  "divide": "div.rn.f64", "maximum": "max.f64", "minimum": "min.f64"}
        if op in simple:
            k(f"{simple[op]} {d}, {a[0]}, {a[1]};")
        elif op in ("copy", "pad"):
            k(f"mov.f64 {d}, {a[0]};")
        elif op in ("neg", "negative"):
            k(f"neg.f64 {d}, {a[0]};")
        elif op in ("abs", "fabs"):
            k(f"abs.f64 {d}, {a[0]};")
        elif op == "relu":
            k(f"max.f64 {d}, {a[0]}, {f64_hex(0)};")
        elif op == "sqrt":
            k(f"sqrt.rn.f64 {d}, {a[0]};")
        elif op == "reciprocal":
            k(f"rcp.rn.f64 {d}, {a[0]};")
        elif op == "square":
            k(f"mul.rn.f64 {d}, {a[0]}, {a[0]};")
        elif op in ("fma", "mul_add"):
            k(f"fma.rn.f64 {d}, {a[0]}, {a[1]}, {a[2]};")
        else:
            f = [self.convert(x, "f64", "f32") for x in a]
            r = self._op_f32(op, f)
            return self.convert(r, "f32", "f64")
        return d

    def _op_int(self, op, ty, a):
        k = self.k
        pt = PTY[ty]
        cls = REG[ty]
        d = k.reg(cls)
        b = "b64" if cls == "rd" else "b32"
        simple = {"add": f"add.{pt}", "subtract": f"sub.{pt}", "multiply": f"mul.lo.{pt}",
                  "divide": f"div.{pt}", "floor_divide": f"div.{pt}", "maximum": f"max.{pt}",
                  "minimum": f"min.{pt}", "bitwise_and": f"and.{b}", "bitwise_or": f"or.{b}",
                  "bitwise_xor": f"xor.{b}", "mod": f"rem.{pt}", "remainder": f"rem.{pt}",
                  "fmod": f"rem.{pt}", "left_shift": f"shl.{b}",
                  "right_shift": f"shr.{pt}"}
        if op in simple:
            sh = a[1]
            if op in ("left_shift", "right_shift") and cls == "rd":
                t = k.reg("r")
                k(f"cvt.u32.u64 {t}, {a[1]};")
                sh = t
            k(f"{simple[op]} {d}, {a[0]}, {sh};")
        elif op in ("copy", "pad"):
            k(f"mov.{b} {d}, {a[0]};")
        elif op in ("neg", "negative"):
            k(f"neg.{pt if pt[0] == 's' else 's' + pt[1:]} {d}, {a[0]};")
        elif op in ("abs", "fabs"):
            k(f"abs.{pt if pt[0] == 's' else 's' + pt[1:]} {d}, {a[0]};")
        elif op == "square":
            k(f"mul.lo.{pt} {d}, {a[0]}, {a[0]};")
        elif op == "relu":
            k(f"max.{pt} {d}, {a[0]}, 0;")
        elif op == "bitwise_not":
            k(f"not.{b} {d}, {a[0]};")
        else:
            raise NotImplementedError(f"op {op} ({ty})")
        return d


def I_Var(name):
    from .ir import NODE_CLASSES
    return NODE_CLASSES["Var"](name)


class _StepMark:
    """An internal statement at the start / end of a carrying loop's body."""

    def __init__(self, cells, begin):
        self.cells, self.begin = cells, begin


def _is_imm(x) -> bool:
    return isinstance(x, str) and (x.lstrip("-").isdigit())


def _fold(op, a, b):
    if op == "+":
        return a + b
    if op == "-":
        return a - b
    if op == "*":
        return a * b
    if op == "/":
        return int(a / b) if b else 0
    if op == "//":
        return a // b if b else 0
    if op == "%":
        return a - int(a / b) * b if b else 0
    if op == "<<":
        return a << b
    if op == ">>":
        return a >> b
    if op == "&":
        return a & b
    if op == "|":
        return a | b
    if op == "^":
        return a ^ b
    if op == "min":
        return min(a, b)
    if op == "max":
        return max(a, b)
    raise NotImplementedError(op)

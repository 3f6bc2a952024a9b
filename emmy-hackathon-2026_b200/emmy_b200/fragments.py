"""The register-fragment tensor-core statements (``mma.sync``) on sm_100a.

The Kernel IR vocabulary defines, and no reference IR uses, a family of
statements that drive the warp-level ``mma.sync`` instructions through
per-thread register fragments (reference ``TASK.md:143-162``):
``RegFragment`` declares a fragment array, ``LdmatrixLoad`` fills an A or B
fragment, ``MmaSyncPtx`` issues ``c = a . b + c``, ``FragmentApply``,
``FragmentRowReduce``, ``FragmentRepack`` and ``FragmentPromote`` work on
fragments in registers, and ``RegStore`` writes a C fragment to a buffer,
through an optional ``Lambda`` epilogue.  The reference compiler exits 1 on
all of them.  The table names their fields and leaves the fragment geometry
(``FragLayout``) to Emmy; with no serialised example to follow, this module
fixes the forms below, and the IRs in ``synth`` (``mma_matmul``,
``mma_attention``) are written in them:

* a fragment reference is a string: ``"name"`` (the cell ``fragment_index``
  selects, else cell 0) or ``"name[i]"`` with a literal cell ``i``;
* ``shape`` is ``"m16n8k16"`` / ``"m16n8k8"`` or the tuple ``(16, 8, 16)``;
* every fragment holds its elements where the PTX ISA's mma.sync fragment
  figures put them (lane = 4 * group + thread-in-group): A of m16n8k16 16-bit
  holds (g, 2t..2t+1), (g+8, 2t..), (g, 2t+8..), (g+8, 2t+8..); B holds
  (k = 2t..2t+1, n = g), (k = 2t+8.., n = g); the f32 C holds (g, 2t),
  (g, 2t+1), (g+8, 2t), (g+8, 2t+1); tf32 m16n8k8 A holds (g, t), (g+8, t),
  (g, t+4), (g+8, t+4) and B (k = t, n = g), (k = t+4, n = g).  A
  ``FragLayout`` given to ``FragmentApply`` / ``FragmentRowReduce`` /
  ``RegStore`` overrides the C element coordinates (``lane_decl``
  expressions over ``lane`` bind ``lane_names``; ``row_off`` / ``col_off``
  are per-element expressions over them; ``elem_row`` says which of the
  row pair an element belongs to; ``reduce_xors`` are the lane masks of a
  row's reduction);
* ``LdmatrixLoad.src_index`` is the coordinate of the tile's first element in
  its buffer and ``ldm`` the row pitch in elements (default: the buffer's last
  extent).  A is read as ``[m][k]``; B as ``[k][n]`` when ``b_trans`` is true
  (``ldmatrix .trans``) and as ``[n][k]`` otherwise.  A shared-memory source of
  the fragment's own 16-bit type with no guard goes through ``ldmatrix``
  (each row of the 8x8 matrices 16-byte aligned: the IR's pitch and origin
  must keep it so); anything else -- global memory, f32 sources (tf32 or
  converted), ``gmem_guard`` = (row bound, column bound) of the source and
  ``k_zero`` = the bound of the contraction coordinate -- loads element by
  element, zero where a guard fails.  ``swizzle`` (shared memory only) is the
  vocabulary's chunk swizzle of ``CpAsyncCopy`` (``"B128"`` / ``"B64"`` /
  ``"B32"``, optional ``@shift``) applied to every flat element index, so a
  tile copied in swizzled is read back in place;
* ``FragmentApply`` computes ``out = post(op(args))`` per C element; an
  argument is, by ``kinds``: ``frag`` (a fragment reference), ``row`` (a
  (top, bottom) pair of names from ``FragmentRowReduce``), ``scalar`` (a name
  or literal), ``mask`` (a predicate over ``Var("row")`` / ``Var("col")``, the
  element's coordinates ``row_base + row offset``, ``col_base + col offset``;
  1.0 where it holds, else 0.0) or ``bias`` (a (buffer, index) pair read at
  those coordinates);
* ``FragmentRowReduce`` folds the C elements of each row of the pair over the
  listed fragments and then across the lanes that share the row;
* ``FragmentRepack`` packs C fragments ``srcs[2*part]`` and
  ``srcs[2*part+1]`` (columns 0-7 and 8-15 of a 16-column slab) into one
  m16n8k16 A fragment of ``ab_dtype``;
* ``RegStore`` writes each C element to ``dst_index`` with the element's row
  and column offsets added on ``row_dim`` / ``col_dim`` (default the last two
  coordinates; ``ldm``, when given, is the row pitch), only where
  ``row < m_guard`` and ``col < n_guard``; the epilogue ``Lambda`` binds its
  parameters to the element of ``frag`` and of each of ``extra_frags`` and
  ``row`` / ``col`` to the coordinates, runs its body and stores
  ``results[0]``, converted to the buffer's type (``red.add`` when atomic);
  into shared memory it takes the same ``swizzle``.

``LdmatrixLoad.staged`` and ``FragmentApply.in_place`` are accepted and change
nothing: the source buffer's memory space decides how a fragment is loaded,
and an applied fragment's registers are always updated where they are.

Not lowered (exit 1, ``unsupported construct``): ``BlockScaleLoad`` and the
block-scaled ``MmaSyncPtx`` (``sfa_frag`` / ``sfb_frag``) -- block-scaled
``mma.sync`` is an sm_120a instruction, sm_100a scales only through
``tcgen05.mma``; the ``byte_slab`` dequantising and ``pair_frag`` loads;
``volta_interleaved`` stores; swizzled global accesses.
"""
from __future__ import annotations

import re

from .analysis import kind
from .ptx import f32_hex

_SHAPES = {"m16n8k16": (16, 8, 16), "m16n8k8": (16, 8, 8)}
_WIDE = ("bf16", "f16")

# (role, k, operand class) -> [(register, half or None, row (g, t, c), col (g, t, c))]
# coordinates are a*g + b*t + c with g = lane >> 2, t = lane & 3; B's "row"
# is its k coordinate and its "col" its n coordinate
_LAYOUTS: dict = {}


def _build_layouts():
    c32 = [(0, None, (1, 0, 0), (0, 2, 0)), (1, None, (1, 0, 0), (0, 2, 1)),
           (2, None, (1, 0, 8), (0, 2, 0)), (3, None, (1, 0, 8), (0, 2, 1))]
    c16 = [(0, 0, (1, 0, 0), (0, 2, 0)), (0, 1, (1, 0, 0), (0, 2, 1)),
           (1, 0, (1, 0, 8), (0, 2, 0)), (1, 1, (1, 0, 8), (0, 2, 1))]
    for kk in (8, 16):
        _LAYOUTS[("c", kk, "f32")] = c32
        _LAYOUTS[("c", kk, "f16")] = c16
    _LAYOUTS[("a", 16, "wide")] = [(r, h, (1, 0, r0), (0, 2, c0 + h))
                                   for r, (r0, c0) in enumerate([(0, 0), (8, 0), (0, 8), (8, 8)])
                                   for h in (0, 1)]
    _LAYOUTS[("a", 8, "wide")] = [(r, h, (1, 0, r0), (0, 2, h))
                                  for r, r0 in enumerate([0, 8]) for h in (0, 1)]
    _LAYOUTS[("a", 8, "tf32")] = [(r, None, (1, 0, r0), (0, 1, c0))
                                  for r, (r0, c0) in enumerate([(0, 0), (8, 0), (0, 4), (8, 4)])]
    _LAYOUTS[("b", 16, "wide")] = [(r, h, (0, 2, k0 + h), (1, 0, 0))
                                   for r, k0 in enumerate([0, 8]) for h in (0, 1)]
    _LAYOUTS[("b", 8, "wide")] = [(0, h, (0, 2, h), (1, 0, 0)) for h in (0, 1)]
    _LAYOUTS[("b", 8, "tf32")] = [(r, None, (0, 1, k0), (1, 0, 0)) for r, k0 in enumerate([0, 4])]


_build_layouts()


def _dtname(d) -> str:
    if d is None:
        return ""
    n = getattr(d, "name", d)
    return {"float32": "f32", "float16": "f16", "bfloat16": "bf16", "half": "f16"}.get(str(n), str(n))


def _shape(s) -> tuple:
    if isinstance(s, str):
        if s not in _SHAPES:
            raise NotImplementedError(f"mma.sync shape {s}")
        return _SHAPES[s]
    t = tuple(int(x) for x in s)
    if t not in _SHAPES.values():
        raise NotImplementedError(f"mma.sync shape {t}")
    return t


def _cls(dt: str) -> str:
    if dt in _WIDE:
        return "wide"
    if dt == "tf32":
        return "tf32"
    if dt in ("f32", "f16"):
        return dt
    raise NotImplementedError(f"fragment type {dt}")


class Frag:
    def __init__(self, role, shape, dt, cells):
        self.role, self.shape, self.dt, self.cells = role, shape, dt, cells

    def layout(self):
        key = (self.role, self.shape[2], self.dt if self.role == "c" else _cls(self.dt))
        lay = _LAYOUTS.get(key)
        if lay is None:
            raise NotImplementedError(f"{self.role} fragment of {self.dt} for shape {self.shape}")
        return lay

    def nregs(self) -> int:
        return max(r for r, *_ in self.layout()) + 1


class FragmentLowering:
    """Mixin of ``GenericLowering``: the ``s_<statement>`` methods of the
    fragment vocabulary, on the generic lowering's registers and addressing."""

    # ------------------------------------------------------------ helpers
    def _frag_state(self):
        if not hasattr(self, "frags"):
            self.frags = {}
        return self.frags

    def _lane_gt(self):
        """(g, t) = (lane >> 2, lane & 3), computed where a statement needs
        them (a register made inside one branch is undefined in another)."""
        k = self.k
        lane = self.ints["lane"]
        g, t = k.reg("r"), k.reg("r")
        k(f"shr.u32 {g}, {lane}, 2;")
        k(f"and.b32 {t}, {lane}, 3;")
        return g, t

    def _ref(self, ref, index=None):
        frags = self._frag_state()
        m = re.fullmatch(r"\s*([A-Za-z_][\w]*)\s*(?:\[\s*(\d+)\s*\])?\s*", str(ref))
        if not m:
            raise NotImplementedError(f"fragment reference {ref!r}")
        name, cell = m.group(1), m.group(2)
        if name not in frags:
            raise NotImplementedError(f"fragment {name} used before its RegFragment")
        f = frags[name]
        if cell is None:
            cell = 0
            if index is not None:
                if kind(index) == "Literal":
                    cell = int(index.value)
                elif isinstance(index, int):
                    cell = index
                else:
                    raise NotImplementedError("fragment_index must be a literal")
        cell = int(cell)
        if not 0 <= cell < len(f.cells):
            raise NotImplementedError(f"fragment cell {name}[{cell}] out of range")
        return f, f.cells[cell]

    def _coord(self, g, t, abc) -> str:
        a, b, c = abc
        k = self.k
        if a == 0 and b == 0:
            return str(c)
        r = k.reg("r")
        if a and b:
            k(f"mad.lo.s32 {r}, {g}, {a}, {c};")
            k(f"mad.lo.s32 {r}, {t}, {b}, {r};")
        elif a:
            k(f"mad.lo.s32 {r}, {g}, {a}, {c};")
        else:
            k(f"mad.lo.s32 {r}, {t}, {b}, {c};")
        return r

    def _c_elements(self, frag, layout):
        """[(value getter info, row offset operand, col offset operand, row
        pair index)] of a C fragment's elements, from ``layout`` (a
        ``FragLayout``) or the mma.sync C layout."""
        lay = frag.layout()
        if layout is None:
            g, t = self._lane_gt()
            return [(i, self._coord(g, t, r), self._coord(g, t, c), 0 if r[2] < 8 else 1)
                    for i, (_, _, r, c) in enumerate(lay)]
        n = int(layout.n_elems)
        if n != len(lay):
            raise NotImplementedError(f"FragLayout of {n} elements for a {len(lay)}-element fragment")
        saved = dict(self.ints)
        names = tuple(layout.lane_names or ())
        decl = tuple(layout.lane_decl or ())
        if len(names) != len(decl):
            raise NotImplementedError("FragLayout lane_decl / lane_names lengths differ")
        for nm, e in zip(names, decl):
            self.ints[nm] = self.ival(e)
        out = []
        for i in range(n):
            out.append((i, self.ival(layout.row_off[i]), self.ival(layout.col_off[i]),
                        int(layout.elem_row[i])))
        self.ints = saved
        return out

    def _c_value(self, frag, regs, i) -> str:
        """Element i of a C fragment as an f32 register."""
        k = self.k
        r, h, _, _ = frag.layout()[i]
        if h is None:
            return regs[r]
        lo, hi = k.reg("h"), k.reg("h")
        k(f"mov.b32 {{{lo}, {hi}}}, {regs[r]};")
        f = k.reg("f")
        k(f"cvt.f32.f16 {f}, {hi if h else lo};")
        return f

    def _c_set(self, frag, regs, i, val):
        """Element i of a C fragment := the f32 value ``val``."""
        k = self.k
        r, h, _, _ = frag.layout()[i]
        if h is None:
            k(f"mov.f32 {regs[r]}, {val};")
            return
        x = k.reg("h")
        k(f"cvt.rn.f16.f32 {x}, {val};")
        lo, hi = k.reg("h"), k.reg("h")
        k(f"mov.b32 {{{lo}, {hi}}}, {regs[r]};")
        pair = (lo, x) if h else (x, hi)
        k(f"mov.b32 {regs[r]}, {{{pair[0]}, {pair[1]}}};")

    def _operand(self, name):
        """A named value or a literal as an (f32 register, "f32") pair."""
        k = self.k
        if isinstance(name, (int, float)) or kind(name) == "Literal":
            v = float(getattr(name, "value", name))
            r = k.reg("f")
            k(f"mov.f32 {r}, {f32_hex(v)};")
            return r, "f32"
        if kind(name) == "Var":
            name = name.name
        v, ty = self.vals[name]
        return self.convert(v, ty, "f32"), "f32"

    def _flat_ops(self, index, shape, subst):
        """Flat element offset of ``index`` (expressions) in a buffer of
        ``shape`` with ``subst`` = {dimension: operand to add}."""
        acc = "0"
        for d, e in enumerate(index):
            term = self.ival(e)
            if d in subst:
                term = self._iadd(term, subst[d])
            suffix = 1
            for x in shape[d + 1:]:
                suffix *= int(x)
            if suffix != 1:
                term = self._imul(term, suffix)
            acc = self._iadd(acc, term)
        return acc

    # ------------------------------------------------------------ statements
    def s_RegFragment(self, s):
        k = self.k
        frags = self._frag_state()
        role = str(s.role).lower()[:1]
        if role not in ("a", "b", "c"):
            raise NotImplementedError(f"RegFragment role {s.role!r}")
        shape = _shape(s.shape)
        dt = _dtname(s.dtype) or ("f32" if role == "c" else "bf16")
        count = int(s.count or 1)
        probe = Frag(role, shape, dt, [])
        n = probe.nregs()
        if s.nregs is not None and int(s.nregs) != n:
            raise NotImplementedError(f"RegFragment {s.name}: {s.nregs} registers, the {role} "
                                      f"fragment of {dt} {shape} has {n}")
        old = frags.get(s.name)
        if old is not None and (old.role, old.shape, old.dt, len(old.cells)) == \
                (role, shape, dt, count):
            # declared again (a loop body's RegFragment): zero the same registers
            cells = old.cells
        else:
            cells = [[k.reg("f" if (role == "c" and dt == "f32") else "r") for _ in range(n)]
                     for _ in range(count)]
        for regs in cells:
            for r in regs:
                k(f"mov.f32 {r}, 0f00000000;" if r.startswith("%f") else f"mov.b32 {r}, 0;")
        frags[s.name] = Frag(role, shape, dt, cells)

    def s_BlockScaleLoad(self, s):
        raise NotImplementedError("BlockScaleLoad: block-scaled mma.sync is an sm_120a "
                                  "instruction; sm_100a scales blocks only in tcgen05.mma")

    def s_LdmatrixLoad(self, s):
        k = self.k
        frag, regs = self._ref(s.frag, s.fragment_index)
        role = str(s.role or frag.role).lower()[:1]
        if role != frag.role or role == "c":
            raise NotImplementedError(f"LdmatrixLoad role {s.role!r} into a {frag.role} fragment")
        for f in ("byte_slab", "scale_buffer", "pair_frag"):
            if getattr(s, f, None):
                raise NotImplementedError(f"LdmatrixLoad {f}")
        if getattr(s, "fragment_layout", None) is not None:
            raise NotImplementedError("LdmatrixLoad with a custom fragment layout")
        src = s.src_buffer
        shared = src in self.smem
        swz = getattr(s, "swizzle", None)
        swz = None if swz in (None, False, "NONE", "none") else swz
        if swz is not None and not shared:
            raise NotImplementedError("LdmatrixLoad swizzle of a global buffer")
        shape = self.shape_of(src)
        sty = self.smem[src]["ty"] if shared else self.ctx.bufs.dtypes.get(src, "f32")
        ldm = int(s.ldm) if s.ldm else int(shape[-1])
        index = tuple(s.src_index)
        if len(index) < 2:
            raise NotImplementedError("LdmatrixLoad src_index needs a row and a column")
        btrans = bool(s.b_trans)
        guard = s.gmem_guard
        kz = s.k_zero
        kk = frag.shape[2]
        base = self.flat(index, shape)
        if shared and sty == frag.dt and frag.dt in _WIDE and guard is None and kz is None:
            # the lane whose address feeds each 8x8 matrix row: A x4 takes
            # matrices (rows 0-7, 8-15) x (k 0-7, 8-15) from lanes 0-31;
            # B [k][n] (.trans) k rows 0-15; B [n][k] n rows 0-7 at k 0 / 8
            lane = self.ints["lane"]
            n = frag.nregs()
            if role == "a":
                row_mask, col_shift, trans = 15, (4 if kk == 16 else None), ""
            elif btrans:
                row_mask, col_shift, trans = (15 if kk == 16 else 7), None, ".trans"
            else:
                row_mask, col_shift, trans = 7, (3 if kk == 16 else None), ""
            r = k.reg("r")
            k(f"and.b32 {r}, {lane}, {row_mask};")
            off = k.reg("r")
            k(f"mul.lo.s32 {off}, {r}, {ldm};")
            if col_shift is not None:
                c = k.reg("r")
                k(f"shr.u32 {c}, {lane}, {col_shift};")
                k(f"and.b32 {c}, {c}, 1;")
                k(f"mad.lo.s32 {off}, {c}, 8, {off};")
            addr = self.saddr(src, self.apply_swizzle(self._iadd(base, off), swz))
            k(f"ldmatrix.sync.aligned.m8n8.x{n}{trans}.shared.b16 "
              f"{{{', '.join(regs)}}}, [{addr}];")
            return
        # element by element
        g, t = self._lane_gt()
        lay = frag.layout()
        orow = self.ival(index[-2])
        ocol = self.ival(index[-1])
        halves: dict = {}
        for (r, h, rc, cc) in lay:
            a = self._coord(g, t, rc)     # A: row;  B: k
            b = self._coord(g, t, cc)     # A: col;  B: n
            if role == "a" or btrans:
                dr, dc = a, b
            else:
                dr, dc = b, a
            kcoord_is_col = role == "a" or not btrans
            off = self._iadd(self._imul(dr, ldm) if not _imm(dr) else str(int(dr) * ldm), dc)
            flat = self.apply_swizzle(self._iadd(base, off), swz)
            p = None
            conds = []
            if guard is not None:
                gr, gc = (tuple(guard) + (None, None))[:2]
                if gr is not None:
                    conds.append((self._iadd(orow, dr), self.ival(gr)))
                if gc is not None:
                    conds.append((self._iadd(ocol, dc), self.ival(gc)))
            if kz is not None:
                kabs = self._iadd(ocol, dc) if kcoord_is_col else self._iadd(orow, dr)
                conds.append((kabs, self.ival(kz)))
            for lhs, rhs in conds:
                q = k.reg("p")
                lhs_r = lhs
                if _imm(lhs):
                    lhs_r = k.reg("r")
                    k(f"mov.b32 {lhs_r}, {lhs};")
                k(f"setp.lt.s32 {q}, {lhs_r}, {rhs};")
                if p is None:
                    p = q
                else:
                    p2 = k.reg("p")
                    k(f"and.pred {p2}, {p}, {q};")
                    p = p2
            pre = f"@{p} " if p is not None else ""
            space = "shared" if shared else "global"
            addr = self.saddr(src, flat) if shared else self.gaddr(src, flat, _nbytes(sty))
            if sty in _WIDE:
                x = k.reg("h")
                k(f"mov.b16 {x}, 0;")
                k(f"{pre}ld.{space}.b16 {x}, [{addr}];")
                if frag.dt == sty:
                    val16 = x
                    valf = None
                else:
                    valf = k.reg("f")
                    k(f"cvt.f32.{sty} {valf}, {x};")
                    val16 = None
            elif sty == "f32":
                valf = k.reg("f")
                k(f"mov.f32 {valf}, 0f00000000;")
                k(f"{pre}ld.{space}.f32 {valf}, [{addr}];")
                val16 = None
            else:
                raise NotImplementedError(f"LdmatrixLoad from a {sty} buffer")
            if frag.dt == "tf32":
                k(f"cvt.rna.tf32.f32 {regs[r]}, {valf};")
                continue
            if val16 is None:
                val16 = k.reg("h")
                k(f"cvt.rn.{frag.dt}.f32 {val16}, {valf};")
            halves.setdefault(r, {})[h] = val16
        for r, hv in halves.items():
            k(f"mov.b32 {regs[r]}, {{{hv[0]}, {hv[1]}}};")

    def s_MmaSyncPtx(self, s):
        if getattr(s, "sfa_frag", None) or getattr(s, "sfb_frag", None):
            raise NotImplementedError("block-scaled MmaSyncPtx: an sm_120a instruction; "
                                      "sm_100a scales blocks only in tcgen05.mma")
        c, cr = self._ref(s.c_frag)
        a, ar = self._ref(s.a_frag)
        b, br = self._ref(s.b_frag)
        shape = _shape(s.shape) if s.shape is not None else a.shape
        ab = _dtname(s.ab_dtype) or a.dt
        cd = _dtname(s.c_dtype) or c.dt
        if (a.role, b.role, c.role) != ("a", "b", "c"):
            raise NotImplementedError("MmaSyncPtx operands must be a, b and c fragments")
        if a.dt != ab or b.dt != ab or c.dt != cd or a.shape != shape or b.shape != shape:
            raise NotImplementedError(f"MmaSyncPtx {shape} {ab}->{cd} over fragments of "
                                      f"{a.dt}/{b.dt}/{c.dt}")
        ok = ((ab in _WIDE and cd == "f32") or (ab == "f16" and cd == "f16")
              or (ab == "tf32" and cd == "f32" and shape[2] == 8))
        if not ok:
            raise NotImplementedError(f"mma.sync {ab} -> {cd}")
        m, n, kk = shape
        self.k(f"mma.sync.aligned.m{m}n{n}k{kk}.row.col.{cd}.{ab}.{ab}.{cd} "
               f"{{{', '.join(cr)}}}, {{{', '.join(ar)}}}, {{{', '.join(br)}}}, "
               f"{{{', '.join(cr)}}};")

    def s_FragmentPromote(self, s):
        k = self.k
        d, dr = self._ref(s.dst)
        f, fr = self._ref(s.src)
        if d.role != "c" or f.role != "c" or d.dt != "f32" or f.dt != "f16":
            raise NotImplementedError("FragmentPromote adds an f16 C fragment into an f32 one")
        for i in range(4):
            v = self._c_value(f, fr, i)
            self._c_set(d, dr, i, _add(k, self._c_value(d, dr, i), v))
        for r in fr:
            k(f"mov.b32 {r}, 0;")

    def s_FragmentApply(self, s):
        k = self.k
        out, outr = self._ref(s.out)
        if out.role != "c":
            raise NotImplementedError("FragmentApply writes a C fragment")
        op = getattr(s.op, "name", s.op)
        post = getattr(s.post, "name", s.post) if s.post else None
        kinds = tuple(s.kinds or ())
        args = tuple(s.args or ())
        if len(kinds) != len(args):
            raise NotImplementedError("FragmentApply args and kinds differ in length")
        elems = self._c_elements(out, s.layout)
        rb = self.ival(s.row_base) if s.row_base is not None else "0"
        cb = self.ival(s.col_base) if s.col_base is not None else "0"
        scalars = {}
        for j, (a, kd) in enumerate(zip(args, kinds)):
            if kd == "scalar":
                scalars[j] = self._operand(a)
        results = []
        for (i, ro, co, half) in elems:
            vals = []
            row = col = None
            for j, (a, kd) in enumerate(zip(args, kinds)):
                if kd == "frag":
                    f, fr = self._ref(a)
                    vals.append((self._c_value(f, fr, i), "f32"))
                elif kd == "row":
                    vals.append(self._operand(tuple(a)[half]))
                elif kd == "scalar":
                    vals.append(scalars[j])
                elif kd in ("mask", "bias"):
                    if row is None:
                        row, col = self._iadd(rb, ro), self._iadd(cb, co)
                    saved = dict(self.ints)
                    self.ints["row"], self.ints["col"] = _reg(k, row), _reg(k, col)
                    if kd == "mask":
                        p = self.pred(a)
                        r = k.reg("f")
                        k(f"selp.f32 {r}, 0f3F800000, 0f00000000, {p};")
                        vals.append((r, "f32"))
                    else:
                        buf, idx = a
                        flat = self.flat(tuple(idx), self.shape_of(buf))
                        vals.append(self._load_f32(buf, flat))
                    self.ints = saved
                else:
                    raise NotImplementedError(f"FragmentApply argument kind {kd!r}")
            r, ty = self.op(op, "f32", vals)
            if post:
                r, ty = self.op(post, "f32", [(r, ty)])
            results.append(self.convert(r, ty, "f32"))
        for (i, *_), r in zip(elems, results):
            self._c_set(out, outr, i, r)

    def s_FragmentRowReduce(self, s):
        k = self.k
        op = str(getattr(s.op, "name", s.op))
        ins = {"max": "max.f32", "maximum": "max.f32", "min": "min.f32", "minimum": "min.f32",
               "add": "add.rn.f32", "sum": "add.rn.f32"}.get(op)
        if ins is None:
            raise NotImplementedError(f"FragmentRowReduce op {op}")
        parts = [None, None]
        xors = (1, 2)
        if s.layout is not None and s.layout.reduce_xors:
            xors = tuple(int(x) for x in s.layout.reduce_xors)
        for ref in tuple(s.frags):
            f, fr = self._ref(ref)
            for (i, _, _, half) in self._c_elements(f, s.layout):
                v = self._c_value(f, fr, i)
                if parts[half] is None:
                    r = k.reg("f")
                    k(f"mov.f32 {r}, {v};")
                    parts[half] = r
                else:
                    r = k.reg("f")
                    k(f"{ins} {r}, {parts[half]}, {v};")
                    parts[half] = r
        for h in (0, 1):
            if parts[h] is None:
                raise NotImplementedError("FragmentRowReduce over no elements of a row")
            for x in xors:
                o = k.reg("f")
                k(f"shfl.sync.bfly.b32 {o}, {parts[h]}, {x}, 31, 0xffffffff;")
                r = k.reg("f")
                k(f"{ins} {r}, {parts[h]}, {o};")
                parts[h] = r
        self.vals[s.top] = (parts[0], "f32")
        self.vals[s.bot] = (parts[1], "f32")

    def s_FragmentRepack(self, s):
        k = self.k
        a, ar = self._ref(s.frag)
        dt = _dtname(s.ab_dtype) or a.dt
        if a.role != "a" or a.dt != dt or dt not in _WIDE or a.shape[2] != 16:
            raise NotImplementedError("FragmentRepack makes a 16-bit m16n8k16 A fragment")
        if getattr(s, "fragment_layout", None) is not None:
            raise NotImplementedError("FragmentRepack with a custom fragment layout")
        part = int(s.part or 0)
        srcs = tuple(s.srcs)
        if len(srcs) < 2 * part + 2:
            raise NotImplementedError("FragmentRepack needs two C fragments per part")
        halves = []
        for ref in srcs[2 * part: 2 * part + 2]:
            f, fr = self._ref(ref)
            if f.role != "c":
                raise NotImplementedError("FragmentRepack reads C fragments")
            halves.append([self._c_value(f, fr, i) for i in range(4)])
        left, right = halves
        # A registers: (g, 2t..), (g+8, 2t..), (g, 2t+8..), (g+8, 2t+8..);
        # cvt.rn.<t>x2.f32 d, hi, lo puts the lower column in the low half
        for reg, (lo, hi) in zip(ar, [(left[0], left[1]), (left[2], left[3]),
                                      (right[0], right[1]), (right[2], right[3])]):
            k(f"cvt.rn.{dt}x2.f32 {reg}, {hi}, {lo};")

    def s_RegStore(self, s):
        k = self.k
        frag, regs = self._ref(s.frag, s.fragment_index)
        if frag.role != "c":
            raise NotImplementedError("RegStore stores a C fragment")
        if getattr(s, "volta_interleaved", False):
            raise NotImplementedError("RegStore volta_interleaved")
        buf = s.dst_buffer
        shared = buf in self.smem
        swz = getattr(s, "swizzle", None)
        swz = None if swz in (None, False, "NONE", "none") else swz
        if swz is not None and not shared:
            raise NotImplementedError("RegStore swizzle into a global buffer")
        shape = self.shape_of(buf)
        ty = self.smem[buf]["ty"] if shared else self.ctx.bufs.dtypes.get(buf, "f32")
        index = tuple(s.dst_index)
        nd = len(index)
        rd = int(s.row_dim) if s.row_dim is not None else nd - 2
        cd = int(s.col_dim) if s.col_dim is not None else nd - 1
        rd, cd = rd % nd, cd % nd
        extras = [self._ref(x) for x in tuple(s.extra_frags or ())]
        elems = self._c_elements(frag, s.fragment_layout)
        orow, ocol = self.ival(index[rd]), self.ival(index[cd])
        for (i, ro, co, _) in elems:
            row, col = _reg(k, self._iadd(orow, ro)), _reg(k, self._iadd(ocol, co))
            skip = k.label("RS_SKIP")
            conds = []
            if s.m_guard is not None:
                conds.append((row, self.ival(s.m_guard)))
            if s.n_guard is not None:
                conds.append((col, self.ival(s.n_guard)))
            for lhs, rhs in conds:
                q = k.reg("p")
                k(f"setp.ge.s32 {q}, {lhs}, {rhs};")
                k(f"@{q} bra {skip};")
            val = self._c_value(frag, regs, i)
            if s.epilogue is not None:
                lam = s.epilogue
                saved_v, saved_i = dict(self.vals), dict(self.ints)
                params = tuple(lam.params)
                binds = [val] + [self._c_value(f, fr, i) for f, fr in extras]
                for p, v in zip(params, binds):
                    self.vals[p] = (v, "f32")
                self.ints["row"], self.ints["col"] = row, col
                self.body(tuple(lam.body))
                res = tuple(lam.results)[0]
                rv, rty = self.vals[res]
                val = self.convert(rv, rty, "f32")
                self.vals, self.ints = saved_v, saved_i
            if s.ldm is not None:
                # origin + row offset * ldm + column offset
                flat = self._iadd(self.flat(index, shape),
                                  self._iadd(self._imul(ro, int(s.ldm)), co))
            else:
                flat = self._flat_ops(index, shape, {rd: ro, cd: co})
            flat = self.apply_swizzle(flat, swz)
            self._store_f32(buf, flat, ty, val, bool(s.atomic), shared)
            k.mark(skip)

    # ------------------------------------------------------------ memory
    def _load_f32(self, buf, flat):
        k = self.k
        shared = buf in self.smem
        ty = self.smem[buf]["ty"] if shared else self.ctx.bufs.dtypes.get(buf, "f32")
        space = "shared" if shared else "global"
        addr = self.saddr(buf, flat) if shared else self.gaddr(buf, flat, _nbytes(ty))
        if ty in _WIDE:
            h = k.reg("h")
            k(f"ld.{space}.b16 {h}, [{addr}];")
            f = k.reg("f")
            k(f"cvt.f32.{ty} {f}, {h};")
            return f, "f32"
        if ty != "f32":
            raise NotImplementedError(f"fragment bias from a {ty} buffer")
        f = k.reg("f")
        k(f"ld.{space}.f32 {f}, [{addr}];")
        return f, "f32"

    def _store_f32(self, buf, flat, ty, val, atomic, shared):
        k = self.k
        space = "shared" if shared else "global"
        addr = self.saddr(buf, flat) if shared else self.gaddr(buf, flat, _nbytes(ty))
        if ty in _WIDE:
            h = k.reg("h")
            k(f"cvt.rn.{ty}.f32 {h}, {val};")
            if atomic:
                k(f"red.{space}.add.noftz.{ty} [{addr}], {h};")
            else:
                k(f"st.{space}.b16 [{addr}], {h};")
        elif ty == "f32":
            k(f"{'red' if atomic else 'st'}.{space}.{'add.' if atomic else ''}f32 [{addr}], {val};")
        else:
            raise NotImplementedError(f"RegStore into a {ty} buffer")


def _imm(x) -> bool:
    return isinstance(x, str) and (x.lstrip("-").isdigit())


def _nbytes(ty: str) -> int:
    return {"f32": 4, "bf16": 2, "f16": 2}.get(ty, 4)


def _reg(k, x) -> str:
    if _imm(x):
        r = k.reg("r")
        k(f"mov.b32 {r}, {x};")
        return r
    return x


def _add(k, a, b) -> str:
    r = k.reg("f")
    k(f"add.rn.f32 {r}, {a}, {b};")
    return r

"""Pointwise template: ``out[e] = f(in_1[e], ..., in_k[e], scalars)`` over a
contiguous f32 domain, as 256-bit vector loads and stores.

Matches the two Emmy schedule forms of a pointwise kernel:

* unrolled cells -- ``Tile[a0..] { U x (Load/Assign) ; Write out[U*cell + c] = (...) }``
  (reference ``problems/p01_vector_add/*.ir.txt:1-8``, lowered by the
  reference's ``compile_tile``/``stmt_load``/``stmt_write``,
  ``compile.py:2469-2534,1207-1271,1315-1386``);
* strided loop -- ``Tile[a0_co] { for a0 in a0_co..N:T { Load/Assign ; Write out[a0] } }``.

The element function ``f`` is recovered from the IR by tracing every written
value back through its ``Assign``/``Load``/``Let`` definitions; the template
only accepts the kernel when every written element has the same function of
"its own" input elements (loads at the written flat offset) and of broadcast
scalars (loads at a constant index), and when the writes cover the output
exactly once.  Those conditions make any partition of the domain over the
launched threads produce the same bytes, so the kernel is free to give each
thread 8 consecutive floats (one ``ld/st.global.v8.f32`` per buffer, 32 B) in
a grid-stride loop that keeps a batch of vectors per buffer in flight: the
batch grows when the IR launches few threads per SM (HBM needs about 128 KB
in flight per SM) and is predicated, so a thread's last, partial batch is one
round trip, not a serial tail.  The
arithmetic uses the ``.rn`` instructions of :mod:`emmy_b200.ops`, so the
result is bit-identical to numpy's float32 evaluation of the same ops.
"""
from __future__ import annotations

from math import prod

from ..analysis import NotAffine, affine, flat_index, kind
from ..ptx import Kernel, f32_hex
from ..ops import emit_op_f32
from .common import (Chain, TemplateMismatch, addr_of, dtype_name, ld_global_f32, linear_ids,
                     pick_vec, st_global_f32)

UNROLL = 4              # smallest batch (vectors per buffer in flight per thread)
UNROLL_MAX = 16
INFLIGHT = 128 * 1024   # bytes of loads in flight per SM that the batch aims for
DATA_REGS = 128         # cap on the batch's loaded registers per thread
SMS = 148


def batch_size(threads: int, inputs: int, vec: int) -> int:
    """Vectors per input buffer each thread keeps in flight: enough for
    INFLIGHT bytes per SM at this launch, a power of two in [UNROLL,
    UNROLL_MAX], and at most DATA_REGS loaded registers."""
    per_sm = max(1, -(-threads // SMS))
    inputs = max(1, inputs)
    u = UNROLL
    while (u * 2 <= UNROLL_MAX and per_sm * inputs * 4 * vec * u < INFLIGHT
           and u * 2 * inputs * vec <= DATA_REGS):
        u *= 2
    return u


class PointwiseTemplate:
    name = "pointwise"

    def __init__(self, ctx, out, n, program, elem_inputs, consts):
        self.ctx = ctx
        self.out = out
        self.n = n
        self.program = program          # canonical element tree
        self.elem_inputs = elem_inputs  # buffers read at the element's own offset
        self.consts = consts            # (buffer, index) broadcast scalars

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "PointwiseTemplate":
        tile = ctx.tile
        if tile is None:
            raise TemplateMismatch("no single top-level Tile")
        if getattr(tile, "aux_threads", 0) or getattr(tile, "raster_group", None):
            raise TemplateMismatch("aux threads / raster")
        axes = ctx.tile_axes()
        body = list(tile.body)
        loops = [s for s in body if kind(s) == "StridedLoop"]
        straight_kinds = {"Load", "Assign", "Let", "Write"}
        bufs = ctx.bufs
        if loops:
            # strided form: pre-statements + exactly one loop, nothing after
            if len(loops) != 1 or body[-1] is not loops[0] or len(axes) != 1:
                raise TemplateMismatch("strided pointwise shape")
            loop = loops[0]
            pre = body[:-1]
            inner = list(loop.body)
            co, T = axes[0]
            if not (kind(loop.start) == "Var" and loop.start.name == co
                    and kind(loop.step) == "Literal" and loop.step.value == T
                    and loop.end is None):
                raise TemplateMismatch("loop does not stride the cooperative axis")
            X = loop.axis.name
            from ..ir import dim
            extent = dim(loop.axis.extent)
            stmts = pre + inner
            domain_vars = [(X, extent)]
        else:
            stmts = body
            domain_vars = axes
        if any(kind(s) not in straight_kinds for s in stmts):
            raise TemplateMismatch("non-straight-line statement")
        writes = [s for s in stmts if kind(s) == "Write"]
        if not writes:
            raise TemplateMismatch("no writes")
        outs = {w.output for w in writes}
        if len(outs) != 1:
            raise TemplateMismatch("more than one output")
        out = outs.pop()
        if bufs.dtypes.get(out) != "f32" or any(w.atomic for w in writes):
            raise TemplateMismatch("output dtype/atomic")
        N = bufs.size(out)
        defs = {}
        for s in stmts:
            if kind(s) == "Load":
                for i, nm in enumerate(s.names):
                    defs[nm] = (s, i)
            elif kind(s) in ("Assign", "Let"):
                defs[s.name] = (s, 0)
        # row-major linear cell index over the domain variables
        strides = {}
        acc = 1
        for name, ext in reversed(domain_vars):
            strides[name] = acc
            acc *= ext
        ncells = acc
        covered = set()
        program = None
        elem_inputs, consts = set(), set()
        U = None
        for w in writes:
            try:
                F = flat_index(w.index, bufs.shapes[out])
            except NotAffine as e:
                raise TemplateMismatch(str(e))
            # F must be U * linear_cell + c
            d = F.as_dict()
            if set(d) - set(strides):
                raise TemplateMismatch("write index uses non-domain variables")
            u = None
            for name, _ in domain_vars:
                c = d.get(name, 0)
                if strides[name] == 0 or c % strides[name]:
                    raise TemplateMismatch("write index not contiguous in cells")
                q = c // strides[name]
                if ncells > 1 and (u is None or u == q):
                    u = q
                elif ncells > 1:
                    raise TemplateMismatch("write index not uniform in cells")
            u = u if u is not None else len(w.values)
            if U is None:
                U = u
            elif U != u:
                raise TemplateMismatch("inconsistent unroll")
            for j, v in enumerate(w.values):
                covered.add(F.const + j)
                tree = cls._canon(v, F.const + j, F, j, defs, bufs, out, elem_inputs, consts, {})
                if program is None:
                    program = tree
                elif tree != program:
                    raise TemplateMismatch("elements compute different functions")
        if not U or covered != set(range(U)) or U * ncells != N:
            raise TemplateMismatch("writes do not cover the output exactly once")
        for b in elem_inputs:
            if bufs.dtypes.get(b) != "f32" or bufs.size(b) != N:
                raise TemplateMismatch("elementwise input dtype/size")
        for b, _ in consts:
            if bufs.dtypes.get(b) != "f32":
                raise TemplateMismatch("scalar input dtype")
        if any(a in ctx.scalar_tys for a in ctx.arg_order):
            raise TemplateMismatch("by-value scalar arguments")
        return cls(ctx, out, N, program, sorted(elem_inputs), sorted(consts))

    @classmethod
    def _canon(cls, name, off, F, j, defs, bufs, out, elem_inputs, consts, memo):
        if name in memo:
            return memo[name]
        if name not in defs:
            raise TemplateMismatch(f"value {name} defined outside the kernel body")
        s, pos = defs[name]
        k = kind(s)
        if k == "Let":
            if kind(s.value) != "Literal":
                raise TemplateMismatch("non-literal Let")
            r = ("lit", float(s.value.value))
        elif k == "Load":
            if dtype_name(s.dtype) != "f32":
                raise TemplateMismatch("load dtype")
            try:
                G = flat_index(s.index, bufs.shapes[s.input])
            except NotAffine as e:
                raise TemplateMismatch(str(e))
            G = G + affine(pos)
            if G.is_const() and not 0 <= G.const < bufs.size(s.input):
                raise TemplateMismatch(f"constant index {G.const} outside {s.input}")
            if G.is_const() and (bufs.size(s.input) == 1 or not F.coefs):
                if not F.coefs and bufs.size(s.input) != 1 and G.const != off:
                    raise TemplateMismatch("scalar-domain load")
                r = ("const", s.input, G.const)
                consts.add((s.input, G.const))
            elif G.coefs == F.coefs and G.const == off:
                r = ("elem", s.input)
                elem_inputs.add(s.input)
            else:
                raise TemplateMismatch(f"load {s.input} is not elementwise")
        elif k == "Assign":
            if dtype_name(s.dtype) not in (None, "f32"):
                raise TemplateMismatch("assign dtype")
            r = ("op", s.op.name, tuple(cls._canon(a, off, F, j, defs, bufs, out, elem_inputs,
                                                   consts, memo) for a in s.args))
        else:
            raise TemplateMismatch(k)
        memo[name] = r
        return r

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        ctx = self.ctx
        k = Kernel(ctx.entry, ctx.params())
        k.comment(f"emmy-b200 template: pointwise, {self.n} f32 elements")
        base = {a: k.param_ptr(a) for a in ctx.arg_order}
        _, _, gid = linear_ids(k, ctx.grid, ctx.block)
        T = ctx.total_threads
        V = pick_vec(self.n, 1)
        NV = self.n // V
        cval = {}
        for b, idx in self.consts:
            a = k.reg("rd")
            k(f"add.s64 {a}, {base[b]}, {4 * idx};")
            r = k.reg("f")
            k(f"ld.global.nc.f32 {r}, [{a}];")
            cval[(b, idx)] = r
        # vectors per thread at most ceil(NV / T): no batch larger than that
        U = min(batch_size(T, len(self.elem_inputs), V), max(1, -(-NV // T)))
        self.batch = U
        v = k.reg("r")
        k(f"mov.u32 {v}, {gid};")
        p = k.reg("p")
        loop, done = k.label("PW"), k.label("DONE")
        k.mark(loop)
        k(f"setp.ge.s32 {p}, {v}, {NV};")
        k(f"@{p} bra {done};")
        self._body(k, base, cval, v, V, T, U, NV)
        k(f"add.s32 {v}, {v}, {U * T};")
        k(f"bra.uni {loop};")
        k.mark(done)
        k("ret;")
        return k.render()

    def _body(self, k, base, cval, v, V, T, unroll, NV):
        """One batch: vector v + u*T for u < unroll, all loads issued before
        the first store.  Vector v exists (the loop tested it); a later one
        past the end loads the last vector instead (in bounds, never stored)
        and its store is predicated off."""
        vals = []
        addrs = []
        preds = []
        for u in range(unroll):
            idx, pu = v, None
            if u:
                idx = k.reg("r")
                k(f"add.s32 {idx}, {v}, {u * T};")
                pu = k.reg("p")
                k(f"setp.lt.s32 {pu}, {idx}, {NV};")
                k(f"min.s32 {idx}, {idx}, {NV - 1};")
            e = k.reg("r")
            k(f"mul.lo.s32 {e}, {idx}, {V};")
            loaded = {}
            for b in self.elem_inputs:
                a = addr_of(k, base[b], e)
                # coherent loads: they cannot move past the batch's stores (which
                # may alias), so ptxas keeps the whole batch in flight, where it
                # sinks read-only (.nc) loads to their uses
                loaded[b] = ld_global_f32(k, a, V, nc=False, hint=".L1::no_allocate")
            vals.append(loaded)
            addrs.append(e)
            preds.append(pu)
        for u in range(unroll):
            outs = []
            for lane in range(V):
                outs.append(self._eval(k, self.program, vals[u], cval, lane, {}))
            a = addr_of(k, base[self.out], addrs[u])
            st_global_f32(k, a, outs, pred=preds[u])

    def _eval(self, k, t, loaded, cval, lane, memo):
        key = t
        if key in memo:
            return memo[key]
        tag = t[0]
        if tag == "lit":
            r = f32_hex(t[1])
        elif tag == "const":
            r = cval[(t[1], t[2])]
        elif tag == "elem":
            r = loaded[t[1]][lane]
        else:
            args = [self._eval(k, a, loaded, cval, lane, memo) for a in t[2]]
            r = emit_op_f32(k, t[1], args)
        memo[key] = r
        return r

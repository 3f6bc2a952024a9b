"""Row template: reductions and fused row operations over f32 rows.

Matches Emmy's cooperative-reduction schedule (reference
``problems/r01_array_sum``, ``r04_row_sum``, ``f01_rmsnorm``, ``f02_row_softmax``,
``f03_l2norm`` and the split form ``tests/hsx/sum_big``)::

    Tile[row?, co] {                       # one CTA of B threads per row
      pre: Let / Load scalar / Assign
      for X in co..L:B { Load / Assign / Accum }        # pass 1
      WarpShuffle(accs) ; Smem ; if lane==0: smem[warp]=acc ; Sync ; TreeHalve
      post: Load scalar / Assign
      (if co == 0: ... ; out[row] (+)= v)               # reduction
      | (for X in co..L:B { Load / Assign ; out[row, X] = v })   # fused pass 2
    }

The reference lowers these statement by statement (``emit_loop``
``compile.py:1867-2013``, ``stmt_warp_shuffle`` ``:1783-1812``,
``stmt_tree_halve`` ``:1814-1857``), so pass 2 re-reads the row from global
memory and every load is a scalar 4-byte access.  This template keeps the
IR's arithmetic -- the loop bodies, the shuffle combine and the tree combine
are the IR's own ``Assign``/``Accum`` statements, run by :class:`Chain` -- and
replaces the memory schedule:

* thread ``t`` owns ``J`` vectors of ``V`` consecutive columns
  (``V`` up to 8, one 256-bit ``ld.global.nc.v8.f32`` each), all issued before
  any arithmetic;
* when a thread's share is at most 64 values the row stays in registers and
  pass 2 reuses them, so the row is read from HBM exactly once;
* the cross-warp combine loads the per-warp partials into one warp and folds
  them with the IR's combine statements over a shuffle butterfly, in every
  warp at once, so the result is broadcast without a second barrier;
* a split reduction (``Write ... atomic=True`` from every CTA) keeps the
  IR's one ``red.global.add.f32`` per CTA.

Accumulation order differs from the reference (each thread folds its own
columns); reductions are checked at the problems' relative tolerance.
"""
from __future__ import annotations

from math import prod

from ..analysis import NotAffine, affine, cond_var_eq, flat_index, kind
from ..ir import dim
from ..ops import emit_op_f32
from ..ptx import Kernel, f32_hex
from .common import (Chain, TemplateMismatch, accum_identity, addr_of, dtype_name,
                     ld_global_f32, pick_vec, st_global_f32)

RESIDENT_MAX = 64      # values per thread kept in registers across passes
BATCH = 4              # vectors per buffer in flight in the streaming loop
# a launch of fewer CTAs than the B200 has SMs (the open problems' one-CTA
# sums and means) is bound by DRAM round trips per thread, not by bandwidth;
# ptxas keeps only a few register loads of a batch in flight (it places each
# load next to its use), so these launches stage each batch through shared
# memory with cp.async instead -- every copy of a batch in flight at once --
# in at most this many bytes of static shared memory
SMALL_LAUNCH_STAGE = 32 * 1024
# ... or, for a single row-contiguous input, through a ring of this many
# shared-memory stages of at most BULK_STAGE bytes each, each filled by one
# 1-D bulk copy (``cp.async.bulk``, the copy engine: no tensor map, no
# multicast) that one thread issues as soon as every thread has read the
# stage's previous batch: several batches stream in while the threads
# reduce an earlier one (0 stages: the cp.async form).  Measured on one B200
# (same process, alternating, outputs checked): r02 (256 KiB, one CTA)
# 10.6 -> 8.75 us; r03 (128 KiB) 8.58 -> 8.54 us
BULK_STAGES = 3
BULK_STAGE = 15 * 1024


def _lit(e, v=None):
    return kind(e) == "Literal" and (v is None or e.value == v)


def _online_max_sum(body, post_names):
    """Recognise the online (max, sum of exponentials) accumulation of a
    softmax in a pass-1 body (Emmy's form, reference
    ``problems/f02_row_softmax/k_softmax_05263d.ir.txt:1-27``)::

        gn = maximum(A, v); alpha = exp(A - gn); beta = exp(v - gn)
        S = S * alpha + beta * w            # Accum add, base = S * alpha
        A = maximum(A, v)                   # Accum maximum

    with ``v`` and ``w`` computed without A or S.  Folding every element this
    way gives A = max(v) and S = sum(exp(v - A) * w) (the rescaling
    telescopes), which the template evaluates as a max tree followed by
    independent exponentials instead of one dependent chain through every
    element.  Returns None when the body has any other shape."""
    defs = {}
    for st in body:
        k = kind(st)
        if k == "Assign":
            defs[st.name] = st
        elif k == "Let":
            defs[st.name] = st
    accums = [st for st in body if kind(st) == "Accum"]
    if len(accums) != 2:
        return None
    amax = [a for a in accums if a.op.name == "maximum" and not a.base]
    asum = [a for a in accums if a.op.name == "add" and a.base]
    if len(amax) != 1 or len(asum) != 1:
        return None
    A, S, v = amax[0].name, asum[0].name, amax[0].value
    accs = {A, S}

    def deps(name, seen=None):
        seen = set() if seen is None else seen
        if name in accs:
            return {name}
        st = defs.get(name)
        if st is None or kind(st) != "Assign" or name in seen:
            return set()
        seen.add(name)
        out = set()
        for a in st.args:
            out |= deps(a, seen)
        return out

    def op_of(name, op, n):
        st = defs.get(name)
        if st is None or kind(st) != "Assign" or st.op.name != op or len(st.args) != n:
            return None
        return list(st.args)

    sa, sb = op_of(asum[0].base, "multiply", 2), op_of(asum[0].value, "multiply", 2)
    if not sa or not sb or S not in sa:
        return None
    alpha = sa[1 - sa.index(S)]
    dg = op_of(alpha, "exp", 1)
    sub = dg and op_of(dg[0], "subtract", 2)
    if not sub or sub[0] != A:
        return None
    gn = sub[1]
    mx = op_of(gn, "maximum", 2)
    if not mx or sorted(mx) != sorted([A, v]):
        return None
    for i, beta in enumerate(sb):
        w = sb[1 - i]
        e = op_of(beta, "exp", 1)
        d = e and op_of(e[0], "subtract", 2)
        if d and d == [v, gn] and not deps(w):
            break
    else:
        return None
    if deps(v):
        return None
    pattern = {gn, alpha, dg[0], beta, e[0], asum[0].base, asum[0].value}
    if pattern & post_names:
        return None
    pre = [st for st in body if kind(st) != "Accum"
           and not (kind(st) == "Assign" and (st.name in pattern or deps(st.name)))]
    return {"max": A, "sum": S, "v": v, "w": w, "pre": pre}


class RowsTemplate:
    name = "rows"

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "RowsTemplate":
        tile = ctx.tile
        if tile is None:
            raise TemplateMismatch("no single top-level Tile")
        if getattr(tile, "aux_threads", 0) or getattr(tile, "raster_group", None):
            raise TemplateMismatch("aux threads / raster")
        axes = ctx.tile_axes()
        if len(axes) == 1:
            row_ax, R = None, 1
            co, B = axes[0]
        elif len(axes) == 2:
            (row_ax, R), (co, B) = axes
        else:
            raise TemplateMismatch("row tile rank")
        if ctx.block != (B, 1, 1) or ctx.grid[0] * ctx.grid[1] * ctx.grid[2] != R:
            raise TemplateMismatch("launch is not one CTA per row")
        if B % 32 or B > 1024:
            raise TemplateMismatch("row threads not a warp multiple")
        body = list(tile.body)
        i = 0
        pre = []
        while i < len(body) and kind(body[i]) in ("Let", "Load", "Assign"):
            pre.append(body[i])
            i += 1
        if i >= len(body) or kind(body[i]) != "StridedLoop":
            raise TemplateMismatch("no pass-1 loop")
        loop1 = body[i]
        i += 1
        L = cls._check_loop(loop1, co, B)
        if i >= len(body) or kind(body[i]) != "WarpShuffle":
            raise TemplateMismatch("no warp shuffle")
        ws = body[i]
        i += 1
        if ws.length != 32:
            raise TemplateMismatch("sub-warp shuffle")
        smems = {}
        while i < len(body) and kind(body[i]) == "Smem":
            smems[body[i].name] = body[i]
            i += 1
        if not (i < len(body) and kind(body[i]) == "Cond" and cond_var_eq(body[i].cond, "lane", 0)):
            raise TemplateMismatch("no lane-0 partial store")
        i += 1
        if not (i < len(body) and kind(body[i]) == "Sync"):
            raise TemplateMismatch("no barrier")
        i += 1
        tree = None
        if i < len(body) and kind(body[i]) == "TreeHalve":
            tree = body[i]
            i += 1
            if tree.length != B // 32 or tree.inner is not None or tree.tid_var != "warp":
                raise TemplateMismatch("tree shape")
            if tuple(tree.state) != tuple(ws.state):
                raise TemplateMismatch("tree and shuffle states differ")
        elif B != 32:
            raise TemplateMismatch("no tree for a multi-warp row")
        post = []
        while i < len(body) and kind(body[i]) in ("Let", "Load", "Assign"):
            post.append(body[i])
            i += 1
        rest = body[i:]
        reduce_tail = loop2 = None
        if len(rest) == 1 and kind(rest[0]) == "Cond" and cond_var_eq(rest[0].cond, co, 0) \
                and not rest[0].else_body:
            reduce_tail = list(rest[0].body)
        elif len(rest) == 1 and kind(rest[0]) == "StridedLoop":
            loop2 = rest[0]
            if cls._check_loop(loop2, co, B) != L:
                raise TemplateMismatch("pass-2 extent differs")
        else:
            raise TemplateMismatch("row tail shape")
        accs = [s for s in loop1.body if kind(s) == "Accum"]
        if [a.name for a in accs] != list(dict.fromkeys(a.name for a in accs)) or \
                set(a.name for a in accs) != set(ws.state):
            raise TemplateMismatch("accumulators differ from shuffle states")
        for a in accs:
            if dtype_name(a.dtype) != "f32" or a.op.name not in ("add", "maximum", "minimum",
                                                                  "multiply"):
                raise TemplateMismatch("accumulator type/op")
        if L % B:
            raise TemplateMismatch("row length not a multiple of the row threads")
        self = cls()
        self.ctx, self.row_ax, self.R, self.co, self.B, self.L = ctx, row_ax, R, co, B, L
        self.pre, self.loop1, self.ws, self.tree, self.post = pre, loop1, ws, tree, post
        self.reduce_tail, self.loop2, self.accs = reduce_tail, loop2, accs
        self.V = pick_vec(L, B)
        self.J = L // (self.V * B)
        self._classify_loads()
        later = []
        for st in list(post) + list(loop2.body if loop2 is not None else reduce_tail or []):
            later += list(getattr(st, "args", ()) or ()) + list(getattr(st, "values", ()) or ())
        self.online = _online_max_sum(loop1.body, set(later))
        return self

    @staticmethod
    def _check_loop(loop, co, B) -> int:
        if not (kind(loop.start) == "Var" and loop.start.name == co and _lit(loop.step, B)
                and loop.end is None):
            raise TemplateMismatch("loop does not stride the row threads")
        return dim(loop.axis.extent)

    def _classify_loads(self):
        """Sort every Load into element / column / scalar reads."""
        bufs = self.ctx.bufs
        self.load_kind = {}     # id(Load) -> ("elem", buf) | ("col", buf) | ("const", buf, idx)
        rowvars = {self.row_ax} if self.row_ax else set()

        def classify(s, loopvar):
            if dtype_name(s.dtype) != "f32" or bufs.dtypes.get(s.input) != "f32":
                raise TemplateMismatch("load dtype")
            if len(s.names) != 1:
                raise TemplateMismatch("vector load in a row kernel")
            try:
                G = flat_index(s.index, bufs.shapes[s.input])
            except NotAffine as e:
                raise TemplateMismatch(str(e))
            d = G.as_dict()
            if not d:
                if not 0 <= G.const < bufs.size(s.input):
                    raise TemplateMismatch(f"constant index {G.const} outside {s.input}")
                self.load_kind[id(s)] = ("const", s.input, G.const)
                return
            if loopvar is None or G.const != 0 or d.get(loopvar) != 1:
                raise TemplateMismatch(f"load {s.input} is not a row read")
            others = {v: c for v, c in d.items() if v != loopvar}
            if not others:
                if bufs.size(s.input) != self.L:
                    raise TemplateMismatch("column vector size")
                self.load_kind[id(s)] = ("col", s.input)
            elif set(others) <= rowvars and others.get(self.row_ax) == self.L:
                if bufs.size(s.input) != self.R * self.L:
                    raise TemplateMismatch("row buffer size")
                self.load_kind[id(s)] = ("elem", s.input)
            else:
                raise TemplateMismatch(f"load {s.input} index shape")

        for s in self.pre + self.post + (self.reduce_tail or []):
            if kind(s) == "Load":
                classify(s, None)
        for s in self.loop1.body:
            if kind(s) == "Load":
                classify(s, self.loop1.axis.name)
            elif kind(s) not in ("Let", "Assign", "Accum"):
                raise TemplateMismatch(f"{kind(s)} in pass 1")
        self.writes2 = []
        if self.loop2 is not None:
            for s in self.loop2.body:
                if kind(s) == "Load":
                    classify(s, self.loop2.axis.name)
                elif kind(s) == "Write":
                    self._check_write2(s)
                elif kind(s) not in ("Let", "Assign"):
                    raise TemplateMismatch(f"{kind(s)} in pass 2")
        if self.reduce_tail is not None:
            ws = [s for s in self.reduce_tail if kind(s) == "Write"]
            if len(ws) != 1 or self.reduce_tail[-1] is not ws[0] or len(ws[0].values) != 1:
                raise TemplateMismatch("reduction tail shape")
            w = ws[0]
            out = w.output
            if bufs.dtypes.get(out) != "f32":
                raise TemplateMismatch("output dtype")
            try:
                F = flat_index(w.index, bufs.shapes[out])
            except NotAffine as e:
                raise TemplateMismatch(str(e))
            d = F.as_dict()
            if d and not (set(d) == {self.row_ax} and d[self.row_ax] == 1):
                raise TemplateMismatch("reduction output index")
            if not d and self.R > 1 and not w.atomic:
                raise TemplateMismatch("rows race on one output")
            self.red_write = (w, F)
            for s in self.reduce_tail[:-1]:
                if kind(s) not in ("Let", "Load", "Assign"):
                    raise TemplateMismatch("reduction tail statement")

    def _check_write2(self, w):
        bufs = self.ctx.bufs
        if w.atomic or len(w.values) != 1 or bufs.dtypes.get(w.output) != "f32":
            raise TemplateMismatch("pass-2 write shape")
        try:
            F = flat_index(w.index, bufs.shapes[w.output])
        except NotAffine as e:
            raise TemplateMismatch(str(e))
        d = F.as_dict()
        X = self.loop2.axis.name
        if F.const or d.get(X) != 1 or bufs.size(w.output) != self.R * self.L or \
                (self.R > 1 and d.get(self.row_ax) != self.L) or \
                set(d) - {X, self.row_ax}:
            raise TemplateMismatch("pass-2 write index")
        self.writes2.append(w)

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        ctx = self.ctx
        # a full-sum kernel that also finishes the global sum across GPUs
        # (meta "peer_finish": true; the multi-GPU path's own launch
        # descriptor): four parameters after meta arg_order
        self.peer = bool(ctx.info.get("peer_finish"))
        params = ctx.params()
        if self.peer:
            from ..peer import FUSED_PARAMS
            w = self.red_write[0] if self.reduce_tail is not None else None
            if w is None or not w.atomic or self.red_write[1].as_dict():
                raise NotImplementedError("peer_finish: only the split full sum (one atomic "
                                          "add of a scalar per CTA)")
            params = params + FUSED_PARAMS
        k = self.k = Kernel(ctx.entry, params)
        if self.peer:
            k.directive("peer " + " ".join(n for n, _ in FUSED_PARAMS))
            k.decl(".global .align 4 .u32 __emmy_done;")
            k.decl(".global .align 4 .u32 __emmy_status;")
        k.comment(f"emmy-b200 template: rows R={self.R} L={self.L} B={self.B} "
                  f"V={self.V} J={self.J} {'fused' if self.loop2 else 'reduce'}")
        self.base = {a: k.param_ptr(a) for a in ctx.arg_order}
        tid = k.special("%tid.x")
        self.tid = tid
        if self.R > 1:
            row = k.special("%ctaid.x")
        else:
            row = None
        self.row = row
        lane = k.reg("r")
        k(f"and.b32 {lane}, {tid}, 31;")
        warp = k.reg("r")
        k(f"shr.u32 {warp}, {tid}, 5;")
        self.lane, self.warp = lane, warp
        self.consts = {}
        env = {}
        chain = Chain(k, env, self._load_scalar)
        chain.run(self.pre)
        # per-row element offset (in elements) of the thread's first vector
        self.row_off = None
        if row is not None:
            ro = k.reg("rd")
            k(f"mul.wide.u32 {ro}, {row}, {self.L * 4};")
            self.row_off = ro
        col0 = k.reg("r")
        k(f"mul.lo.s32 {col0}, {tid}, {self.V};")
        self.col0 = col0
        # accumulators start at their op's identity (the loop is seeded)
        for a in self.accs:
            r = k.reg("f")
            k(f"mov.f32 {r}, {f32_hex(accum_identity(a.op.name))};")
            env[a.name] = r
        resident = self.J * self.V <= RESIDENT_MAX
        elem1 = self._bufs_of(self.loop1.body, "elem")
        col1 = self._bufs_of(self.loop1.body, "col")
        kept = {}
        if resident:
            vecs = {b: [self._vec_load(b, j, "elem", hint=".L1::no_allocate") for j in range(self.J)]
                    for b in elem1}
            cvecs = {b: [self._vec_load(b, j, "col") for j in range(self.J)] for b in col1}
            if self.online:
                self._online_pass1(chain, env, vecs, cvecs)
            else:
                for j in range(self.J):
                    for ln in range(self.V):
                        self._run_elem(chain, env, self.loop1.body, vecs, cvecs, j, ln)
            kept = vecs
        else:
            self._stream_pass1(chain, env, elem1, col1)
        self._combine(chain, env)
        chain.run(self.post)
        if self.reduce_tail is not None:
            self._reduce_tail(chain, env)
        else:
            self._pass2(chain, env, kept)
        k("ret;")
        return k.render()

    def _bufs_of(self, stmts, what):
        out = []
        for s in stmts:
            if kind(s) == "Load":
                lk = self.load_kind[id(s)]
                if lk[0] == what and lk[1] not in out:
                    out.append(lk[1])
        return out

    def _load_scalar(self, s):
        lk = self.load_kind[id(s)]
        if lk[0] != "const":
            raise TemplateMismatch("row read outside a loop")
        return [self._const(lk[1], lk[2])]

    def _const(self, buf, idx):
        key = (buf, idx)
        if key not in self.consts:
            k = self.k
            a = k.reg("rd")
            k(f"add.s64 {a}, {self.base[buf]}, {4 * idx};")
            r = k.reg("f")
            k(f"ld.global.nc.f32 {r}, [{a}];")
            self.consts[key] = r
        return self.consts[key]

    def _vec_addr(self, buf, j_or_reg, what):
        """Address of vector j (python int) or of the column held in a reg."""
        k = self.k
        if isinstance(j_or_reg, int):
            col = k.reg("r")
            k(f"add.s32 {col}, {self.col0}, {j_or_reg * self.B * self.V};")
        else:
            col = j_or_reg
        a = addr_of(k, self.base[buf], col)
        if what == "elem" and self.row_off is not None:
            a2 = k.reg("rd")
            k(f"add.s64 {a2}, {a}, {self.row_off};")
            a = a2
        return a

    def _vec_load(self, buf, j, what, hint=""):
        a = self._vec_addr(buf, j, what)
        return ld_global_f32(self.k, a, self.V, hint=hint)

    def _run_elem(self, chain, env, stmts, vecs, cvecs, j, ln):
        def load(s):
            lk = self.load_kind[id(s)]
            if lk[0] == "const":
                return [self._const(lk[1], lk[2])]
            if lk[0] == "elem":
                return [vecs[lk[1]][j][ln]]
            return [cvecs[lk[1]][j][ln]]
        chain.load = load
        for s in stmts:
            if kind(s) == "Write":
                continue
            chain.stmt(s)
        chain.load = self._load_scalar

    def _online_pass1(self, chain, env, vecs, cvecs):
        """The recognised online (max, sum exp) accumulation over the
        thread's resident elements: v and w per element from the body's
        accumulator-free statements, A = max tree over the identity and the
        v's, S = sum tree of exp(v - A) * w (no dependent chain)."""
        k = self.k
        o = self.online
        vs, ws = [], []
        for j in range(self.J):
            for ln in range(self.V):
                self._run_elem(chain, env, o["pre"], vecs, cvecs, j, ln)
                vs.append(chain.value(o["v"]))
                ws.append(chain.value(o["w"]))

        def tree(vals, op):
            while len(vals) > 1:
                nxt = [emit_op_f32(k, op, [vals[i], vals[i + 1]])
                       for i in range(0, len(vals) - 1, 2)]
                vals = nxt + ([vals[-1]] if len(vals) % 2 else [])
            return vals[0]

        m = tree([env[o["max"]]] + vs, "maximum")
        terms = []
        for v, w in zip(vs, ws):
            d = emit_op_f32(k, "subtract", [v, m])
            e = emit_op_f32(k, "exp", [d])
            terms.append(e if w == f32_hex(1.0) else emit_op_f32(k, "multiply", [e, w]))
        total = tree(terms, "add")
        k(f"mov.f32 {env[o['max']]}, {m};")
        k(f"mov.f32 {env[o['sum']]}, {total};")

    def _stream_pass1(self, chain, env, elem1, col1):
        """Pass 1 for rows too long to keep in registers: a loop over batches
        of BATCH vectors per buffer, all loads of a batch issued first."""
        k = self.k
        J = self.J
        batch = BATCH
        self.stage = None
        per = self.B * self.V * 4
        if (prod(self.ctx.grid) < 148 and len(elem1) + len(col1) == 1 and BULK_STAGES
                and self.V * 4 % 16 == 0 and self.L * 4 % 16 == 0
                and per <= BULK_STAGE and J > BULK_STAGE // per):
            what = "elem" if elem1 else "col"
            self._stream_bulk(chain, env, list(elem1 or col1)[0], what,
                              max(1, BULK_STAGE // per))
            return
        if prod(self.ctx.grid) < 148 and len(elem1) + len(col1) == 1:
            per = self.B * self.V * 4                  # bytes a vector of every thread
            batch = max(1, min(J, SMALL_LAUNCH_STAGE // per))
            if batch > BATCH and self.V * 4 % 16 == 0:
                k.decl(f".shared .align 16 .b8 __emmy_stage[{batch * per}];")
                self.stage = batch
            else:
                batch = BATCH
        nb, rem = divmod(J, batch)
        jreg = k.reg("r")
        k(f"mov.u32 {jreg}, {self.col0};")
        step = self.B * self.V
        if nb:
            cnt = k.reg("r")
            k(f"mov.u32 {cnt}, 0;")
            top = k.label("ROWS_BATCH")
            k.mark(top)
            self._batch(chain, env, elem1, col1, jreg, batch, step)
            k(f"add.s32 {jreg}, {jreg}, {batch * step};")
            k(f"add.s32 {cnt}, {cnt}, 1;")
            p = k.reg("p")
            k(f"setp.lt.s32 {p}, {cnt}, {nb};")
            k(f"@{p} bra.uni {top};")
        if rem:
            self._batch(chain, env, elem1, col1, jreg, rem, step)

    def _status(self):
        """Register holding the address of ``__emmy_status`` (declared once)."""
        k = self.k
        if not getattr(self, "_status_declared", False) and not self.peer:
            k.decl(".global .align 4 .u32 __emmy_status;")
        self._status_declared = True
        st = k.reg("rd")
        k(f"mov.u64 {st}, __emmy_status;")
        return st

    def _wait_through(self, bar, parity, status, code):
        """Wait for phase ``parity`` of mbarrier ``bar`` for at most WAIT_NS of
        %globaltimer; on expiry record ``code`` in ``__emmy_status`` and go on
        (the CTA barriers after the wait are then still reached by every
        thread: no thread leaves the batch loop on its own)."""
        from .gemm import WAIT_NS
        k = self.k
        p = k.reg("p")
        top, ok = k.label("BW"), k.label("BW_OK")
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar}], {parity};")
        k(f"@{p} bra {ok};")
        t0 = k.reg("rd")
        k(f"mov.u64 {t0}, %globaltimer;")
        k.mark(top)
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar}], {parity};")
        k(f"@{p} bra {ok};")
        t1 = k.reg("rd")
        k(f"mov.u64 {t1}, %globaltimer;")
        k(f"sub.s64 {t1}, {t1}, {t0};")
        q = k.reg("p")
        k(f"setp.lt.s64 {q}, {t1}, {WAIT_NS};")
        k(f"@{q} bra {top};")
        k(f"st.global.u32 [{status}], {code};")
        k.mark(ok)

    def _stream_bulk(self, chain, env, buf, what, batch):
        """Pass 1 of a small launch over one row-contiguous input (``what``:
        "elem", the CTA's row of it, or "col", a vector every row reads): batch i
        (``batch`` vectors of every thread, contiguous in the row) lands in
        stage i % NST by one ``cp.async.bulk`` issued by thread 0 on the
        stage's mbarrier (expect-tx of its bytes); every thread waits for it,
        reads its own vectors (vector u of thread t at u * B * V * 4 +
        t * V * 4: the row's layout, so one copy serves all threads), runs
        the IR's element statements, and after a CTA barrier thread 0 refills
        the stage with batch i + NST.  Batches are unrolled (a few dozen at
        most for these launches), so stage and parity are constants."""
        k = self.k
        J, B, V = self.J, self.B, self.V
        per = B * V * 4
        sb = batch * per
        nbt = -(-J // batch)
        NST = min(BULK_STAGES, nbt)
        k.decl(f".shared .align 128 .b8 __emmy_bulk[{NST * sb}];")
        k.decl(f".shared .align 8 .b64 __emmy_bulk_full[{NST}];")
        status = self._status()
        stg = k.reg("r")
        k(f"mov.u32 {stg}, __emmy_bulk;")
        full = k.reg("r")
        k(f"mov.u32 {full}, __emmy_bulk_full;")
        mine = k.reg("r")
        k(f"mad.lo.u32 {mine}, {self.tid}, {V * 4}, {stg};")
        gb = self.base[buf]
        if what == "elem" and self.row_off is not None:
            g2 = k.reg("rd")
            k(f"add.s64 {g2}, {gb}, {self.row_off};")
            gb = g2
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {self.tid}, 0;")

        def nvec(i):
            return min(batch, J - i * batch)

        def issue(i):
            """Thread 0: batch i into its stage (the stage's reads are done)."""
            st_, nb_ = i % NST, nvec(i) * per
            sk = k.label("NO_BULK")
            k(f"@!{p0} bra {sk};")
            k("fence.proxy.async.shared::cta;")
            k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{full}+{8 * st_}], {nb_};")
            src = k.reg("rd")
            k(f"add.s64 {src}, {gb}, {i * sb};")
            k(f"cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
              f"[{stg}+{st_ * sb}], [{src}], {nb_}, [{full}+{8 * st_}];")
            k.mark(sk)

        sk0 = k.label("NO_INIT")
        k(f"@!{p0} bra {sk0};")
        for st_ in range(NST):
            k(f"mbarrier.init.shared::cta.b64 [{full}+{8 * st_}], 1;")
        k("fence.mbarrier_init.release.cluster;")
        k.mark(sk0)
        k("bar.sync 0;")
        for i in range(NST):
            issue(i)
        for i in range(nbt):
            st_ = i % NST
            self._wait_through(f"{full}+{8 * st_}", (i // NST) & 1, status, 10)
            vecs = []
            for u in range(nvec(i)):
                regs = k.regs("f", V)
                for h in range(V // 4):
                    k(f"ld.shared.v4.f32 {{{', '.join(regs[4 * h:4 * h + 4])}}}, "
                      f"[{mine}+{st_ * sb + u * per + 16 * h}];")
                vecs.append(regs)
            if i + NST < nbt:
                k("bar.sync 0;")              # every thread has read the stage
                issue(i + NST)
            for u in range(nvec(i)):
                for ln in range(V):
                    self._run_elem(chain, env, self.loop1.body,
                                   {buf: vecs} if what == "elem" else {},
                                   {buf: vecs} if what == "col" else {}, u, ln)

    def _batch(self, chain, env, elem1, col1, jreg, n, step):
        k = self.k
        cols = []
        for u in range(n):
            if u == 0:
                cols.append(jreg)
            else:
                c = k.reg("r")
                k(f"add.s32 {c}, {jreg}, {u * step};")
                cols.append(c)
        if self.stage is not None:
            vecs = {b: self._staged_vectors(b, cols, "elem") for b in elem1}
            cvecs = {b: self._staged_vectors(b, cols, "col") for b in col1}
        else:
            vecs = {b: [ld_global_f32(k, self._vec_addr(b, c, "elem"), self.V,
                                      hint=".L1::no_allocate") for c in cols] for b in elem1}
            cvecs = {b: [ld_global_f32(k, self._vec_addr(b, c, "col"), self.V) for c in cols]
                     for b in col1}
        for u in range(n):
            for ln in range(self.V):
                self._run_elem(chain, env, self.loop1.body, vecs, cvecs, u, ln)

    def _staged_vectors(self, buf, cols, what):
        """The batch's vectors of ``buf`` through shared memory: 16-byte
        ``cp.async`` copies of every vector issued first (this thread's own
        slots: vector u at u * B * V * 4 + tid * V * 4 bytes), one commit and
        wait, then the vectors read back -- each thread reads only what it
        copied, so no barrier is needed; the next batch's copies are issued
        after these reads."""
        k = self.k
        base = k.reg("r")
        k(f"mov.u32 {base}, __emmy_stage;")
        mine = k.reg("r")
        k(f"mad.lo.u32 {mine}, {self.tid}, {self.V * 4}, {base};")
        per = self.B * self.V * 4
        for u, c in enumerate(cols):
            ga = self._vec_addr(buf, c, what)
            for h in range(self.V * 4 // 16):
                k(f"cp.async.cg.shared.global [{mine}+{u * per + 16 * h}], [{ga}+{16 * h}], 16;")
        k("cp.async.commit_group;")
        k("cp.async.wait_group 0;")
        out = []
        for u in range(len(cols)):
            regs = k.regs("f", self.V)
            for h in range(self.V // 4):
                k(f"ld.shared.v4.f32 {{{', '.join(regs[4 * h:4 * h + 4])}}}, "
                  f"[{mine}+{u * per + 16 * h}];")
            out.append(regs)
        return out

    def _combine(self, chain, env):
        """Warp butterfly with the IR's combine statements, then the per-warp
        partials folded by one butterfly over the warps (every warp at once)."""
        k = self.k
        states, states_b = list(self.ws.state), list(self.ws.state_b)
        self._butterfly(chain, env, states, states_b, self.ws.combine_states, 32)
        nw = self.B // 32
        if nw == 1:
            return
        tree = self.tree
        # shared partials: one f32 per warp per state
        smem = []
        for st in states:
            nm = f"__emmy_part_{st}"
            k.decl(f".shared .align 16 .b8 {nm}[{4 * nw}];")
            smem.append(nm)
        p = k.reg("p")
        k(f"setp.eq.u32 {p}, {self.lane}, 0;")
        woff = k.reg("r")
        k(f"shl.b32 {woff}, {self.warp}, 2;")
        for st, nm in zip(states, smem):
            base = k.reg("r")
            k(f"mov.u32 {base}, {nm};")
            a = k.reg("r")
            k(f"add.s32 {a}, {base}, {woff};")
            k(f"@{p} st.shared.f32 [{a}], {chain.value(st)};")
        k("bar.sync 0;")
        # lanes < nw read one partial each, the rest start at the identity
        q = k.reg("p")
        k(f"setp.lt.u32 {q}, {self.lane}, {nw};")
        loff = k.reg("r")
        k(f"shl.b32 {loff}, {self.lane}, 2;")
        ident = {a.name: accum_identity(a.op.name) for a in self.accs}
        for st, nm in zip(states, smem):
            r = k.reg("f")
            k(f"mov.f32 {r}, {f32_hex(ident[st])};")
            base = k.reg("r")
            k(f"mov.u32 {base}, {nm};")
            a = k.reg("r")
            k(f"add.s32 {a}, {base}, {loff};")
            k(f"@{q} ld.shared.f32 {r}, [{a}];")
            env[st] = r
        width = 1
        while width < nw:
            width *= 2
        self._butterfly(chain, env, list(tree.state), list(tree.state_b), tree.combine_states,
                        width)
        # the butterfly leaves the row total in lanes [0, width); every lane
        # needs it (pass 2 runs in all threads), so broadcast lane 0's
        for st in tree.state:
            b = k.reg("r")
            k(f"mov.b32 {b}, {chain.value(st)};")
            k(f"shfl.sync.idx.b32 {b}, {b}, 0, 0x1f, 0xffffffff;")
            r = k.reg("f")
            k(f"mov.b32 {r}, {b};")
            env[st] = r

    def _butterfly(self, chain, env, states, states_b, combine, width):
        k = self.k
        off = width // 2
        while off > 0:
            for st, sb in zip(states, states_b):
                src = chain.value(st)
                b = k.reg("r")
                k(f"mov.b32 {b}, {src};")
                pb = k.reg("r")
                k(f"shfl.sync.bfly.b32 {pb}, {b}, {off}, 0x1f, 0xffffffff;")
                peer = k.reg("f")
                k(f"mov.b32 {peer}, {pb};")
                env[sb] = peer
            chain.run(combine)
            off //= 2

    def _reduce_tail(self, chain, env):
        k = self.k
        done = k.label("DONE")
        p = k.reg("p")
        k(f"setp.ne.u32 {p}, {self.tid}, 0;")
        k(f"@{p} bra {done};")
        chain.run(self.reduce_tail[:-1])
        w, F = self.red_write
        v = chain.value(w.values[0])
        base = self.base[w.output]
        if F.as_dict():
            a = addr_of(k, base, self.row)
        else:
            a = k.reg("rd")
            k(f"add.s64 {a}, {base}, {4 * F.const};")
        if w.atomic:
            k(f"red.global.add.f32 [{a}], {v};")
        else:
            k(f"st.global.f32 [{a}], {v};")
        if self.peer:
            from ..peer import emit_fused_finish
            st = k.reg("rd")
            k(f"mov.u64 {st}, __emmy_status;")
            emit_fused_finish(k, a, prod(self.ctx.grid), st, "__emmy_done")
        k.mark(done)

    def _pass2(self, chain, env, kept):
        k = self.k
        body = self.loop2.body
        elem2 = self._bufs_of(body, "elem")
        col2 = self._bufs_of(body, "col")
        out = self.writes2[0].output
        wval = self.writes2[0].values[0]
        for j in range(self.J):
            vecs = {b: [kept[b][j]] if b in kept else [self._vec_load(b, j, "elem")] for b in elem2}
            cvecs = {b: [self._vec_load(b, j, "col")] for b in col2}
            outs = []
            for ln in range(self.V):
                self._run_elem(chain, env, body, vecs, cvecs, 0, ln)
                outs.append(chain.value(wval))
            a = self._vec_addr(out, j, "elem")
            st_global_f32(k, a, outs)

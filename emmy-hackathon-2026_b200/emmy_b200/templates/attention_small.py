"""Attention template for Emmy's own fp32 attention schedules: tcgen05 MMAs fed
by the CTA's threads, a meta-only launch (no tensor maps).

Emmy's open-set attention problems (reference ``problems/a01_attention``,
``a02_attention_128`` and the corpus ``attn*`` IRs) are 2-D, fp32, with K
given pre-transposed (``kt`` [d, S], reference ``tools/expressions_open.py:91-104``)
and tiny: S <= 256 keys.  Their IR gives each CTA a block of query rows and
of output columns (``Tile[a0_b, a5_b, a0_u, a5_u]``), and each thread a
micro-tile whose scores it recomputes by scalar dot products inside an
online-softmax chain over the keys.  This template keeps the CTA assignment
and computes the CTA's block as

* S = Q Kt: the threads stage 32-column slabs of the CTA's Q rows and of kt
  (transposed into K-major on the way) into the 128-byte-swizzle layout with
  their low tf32 parts (:class:`.gemm_small.Stager`), one thread issues
  3xTF32 ``tcgen05.mma`` into TMEM (M = 128, N = S rounded up to 16);
* the row max of the scaled scores, read back from TMEM by the thread that
  owns the row (TMEM lane);
* per 32-key slab: P = 2^(s c - m) from TMEM into shared memory (K-major
  A operand, with its low parts; keys past S are 0), the slab of V for the
  CTA's columns (transposed into K-major), and O += P V_slab (3xTF32) into a
  second TMEM accumulator; the row sum l on the way;
* O / l to global memory for the CTA's rows and columns.

c = log2(e) / the IR's ``div_c1`` constant: the same softmax(q kt / div) v
as the IR's online recurrence, evaluated two-pass (the max first), which the
rescaling of the recurrence telescopes to.  Every mbarrier wait is bounded
by ``%globaltimer`` and reports through ``__emmy_status``.
"""
from __future__ import annotations

from ..analysis import NotAffine, affine, kind, walk
from ..ir import dim
from ..ptx import Kernel
from .common import TemplateMismatch
from .gemm import GemmTemplate, _desc_hi, idesc_mma
from .gemm_small import SMEM_LIMIT, STATIC_MAX, Stager, block_indices

LOG2E = 1.4426950408889634


def _f32hex(v: float) -> str:
    import struct
    return "%08X" % struct.unpack("<I", struct.pack("<f", float(v)))[0]


class AttentionSmallTemplate:
    name = "attention"

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "AttentionSmallTemplate":
        tile = ctx.tile
        if tile is None:
            raise TemplateMismatch("no single top-level Tile")
        if getattr(tile, "aux_threads", 0):
            raise TemplateMismatch("auxiliary-thread tile")
        axes = ctx.tile_axes()
        if [a for a, _ in axes] != ["a0_b", "a5_b", "a0_u", "a5_u"]:
            raise TemplateMismatch("not a 2-D attention tile")
        ext = dict(axes)
        T = ext["a0_u"] * ext["a5_u"]
        bt = getattr(tile, "block_threads", None)
        if ctx.block != (T, 1, 1) or bt not in (None, T) or T % 32 or T > 1024:
            raise TemplateMismatch("CTA is not the a0_u x a5_u thread block")
        if ctx.grid[0] * ctx.grid[1] * ctx.grid[2] != ext["a0_b"] * ext["a5_b"]:
            raise TemplateMismatch("grid is not one CTA per (row block, column block)")
        body = list(tile.body)
        bufs = ctx.bufs
        keyloops = [s for s in body if kind(s) == "Loop"]
        if len(keyloops) != 1:
            raise TemplateMismatch("expected one key loop")
        kl = keyloops[0]
        key = kl.axis.name
        scale_buf = None
        for s in body:
            if kind(s) == "Load":
                try:
                    if all(affine(i).is_const() for i in s.index) and bufs.size(s.input) == 1:
                        scale_buf = s.input
                except NotAffine:
                    pass
        recips = [s for s in body if kind(s) == "Assign" and s.op.name == "reciprocal"]
        if scale_buf is None or not recips:
            raise TemplateMismatch("no 1/scale constant")
        q = kt = v = None
        dvar = None
        ops = set()
        for s in walk(kl.body):
            kd = kind(s)
            if kd == "Loop":
                dvar = dvar or s.axis.name
                for t in s.body:
                    if kind(t) == "Load":
                        fv = [i.free_vars() if hasattr(i, "free_vars") else set()
                              for i in t.index]
                        if len(t.index) == 2 and key in fv[1] and s.axis.name in fv[0]:
                            kt = kt or t.input
                            if t.input != kt:
                                raise TemplateMismatch("two key operands")
                        elif len(t.index) == 2 and "a0_u" in fv[0] and s.axis.name in fv[1]:
                            q = q or t.input
                            if t.input != q:
                                raise TemplateMismatch("two query operands")
                        else:
                            raise TemplateMismatch("dot-product load indexing")
            elif kd == "Load":
                fv = [i.free_vars() if hasattr(i, "free_vars") else set() for i in s.index]
                if len(s.index) == 2 and key in fv[0] and "a5_u" in fv[1]:
                    v = v or s.input
                    if s.input != v:
                        raise TemplateMismatch("two value operands")
            elif kd in ("Assign", "Accum"):
                ops.add(s.op.name)
        if not (q and kt and v) or len({q, kt, v}) != 3:
            raise TemplateMismatch("q/kt/v operands")
        if not {"exp", "maximum", "multiply", "add", "subtract"} <= ops or \
                ops - {"exp", "maximum", "multiply", "add", "subtract", "copy"}:
            raise TemplateMismatch(f"softmax chain ops {sorted(ops)}")
        writes = [s for s in body if kind(s) == "Write"]
        outs = {w.output for w in writes}
        if len(outs) != 1 or any(w.atomic for w in writes) or \
                any(kind(s) == "Cond" for s in body):
            raise TemplateMismatch("output")
        out = outs.pop()
        for nm in (q, kt, v, out):
            if bufs.dtypes.get(nm) != "f32" or len(bufs.shapes.get(nm, ())) != 2:
                raise TemplateMismatch("fp32 2-D operands")
        Sq, d = bufs.shapes[q]
        d2, S = bufs.shapes[kt]
        S2, dv = bufs.shapes[v]
        if d2 != d or S2 != S or tuple(bufs.shapes[out]) != (Sq, dv) or dim(kl.axis.extent) != S:
            raise TemplateMismatch("q/kt/v/out shapes")
        BM = BD = mu = nu = None
        cells = set()
        for w in writes:
            try:
                r, c = affine(w.index[0]), affine(w.index[1])
            except NotAffine as e:
                raise TemplateMismatch(f"store index: {e}")
            if r.vars() - {"a0_b", "a0_u"} or c.vars() - {"a5_b", "a5_u"}:
                raise TemplateMismatch("store index variables")
            t4 = (r.coef("a0_b"), r.coef("a0_u"), c.coef("a5_b"), c.coef("a5_u"))
            if BM is None:
                BM, mu, BD, nu = t4
            if t4 != (BM, mu, BD, nu):
                raise TemplateMismatch("stores disagree on the tile")
            for j in range(len(w.values)):
                cells.add((r.const, c.const + j))
        if not mu or not nu or BM != ext["a0_u"] * mu or BD != ext["a5_u"] * nu:
            raise TemplateMismatch("micro-tiles do not tile the CTA block")
        if cells != {(i, j) for i in range(mu) for j in range(nu)}:
            raise TemplateMismatch("stores do not cover each micro-tile once")
        if ext["a0_b"] * BM != Sq or ext["a5_b"] * BD != dv:
            raise TemplateMismatch("blocks do not cover the output exactly")
        warps = T // 32
        if BM > 128 or BM > 32 * min(4, warps) or S > 256 or BD > 256:
            raise TemplateMismatch("block too large")
        self = cls()
        self.ctx, self.q, self.kt, self.v, self.out, self.scale_buf = ctx, q, kt, v, out, scale_buf
        self.Sq, self.d, self.S, self.dv, self.BM, self.BD, self.T = Sq, d, S, dv, BM, BD, T
        self.nb5 = ext["a5_b"]
        self.Sp = -(-S // 16) * 16
        self.BDp = -(-BD // 16) * 16
        self.ocol = -(-self.Sp // 32) * 32
        self.ncols = max(32, 1 << (self.ocol + self.BDp - 1).bit_length())
        if self.ncols > 512:
            raise TemplateMismatch("TMEM columns")
        self.sa = -(-BM // 8) * 1024
        self.sb = max(self.Sp, self.BDp) * 128
        buf = 2 * self.sa + 2 * self.sb
        self.need = max(buf, self.sa + 128 * 128) + 1024 + 64
        avail = min(ctx.smem_bytes, SMEM_LIMIT)
        cap = SMEM_LIMIT if avail > 48 * 1024 else 48 * 1024
        if avail >= self.need:
            self.dynamic = True
        elif self.need <= STATIC_MAX and self.need + avail <= cap:
            self.dynamic = False
        else:
            raise TemplateMismatch("shared memory")
        return self

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        ctx = self.ctx
        T, BM, BD, S, d, Sq, dv = self.T, self.BM, self.BD, self.S, self.d, self.Sq, self.dv
        Sp, BDp, ocol, sa, sb = self.Sp, self.BDp, self.ocol, self.sa, self.sb
        k = Kernel(ctx.entry, ctx.params())
        k.maxntid = (T, 1, 1)
        if self.dynamic:
            k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
        else:
            k.decl(f".shared .align 1024 .b8 __emmy_smem[{self.need}];")
        k.decl(".global .align 4 .u32 __emmy_status;")
        k.comment(f"emmy-b200 template: tcgen05 attention (3xTF32), meta-only launch, "
                  f"q[{Sq},{d}] kt[{d},{S}] v[{S},{dv}], CTA block {BM} rows x {BD} columns, "
                  f"{T} threads")
        qb, kb_, vb, ob = (k.param_ptr(x) for x in (self.q, self.kt, self.v, self.out))
        sbuf = k.param_ptr(self.scale_buf)
        tid = k.special("%tid.x")
        warp = k.reg("r")
        k(f"shr.u32 {warp}, {tid}, 5;")
        lane = k.reg("r")
        k(f"and.b32 {lane}, {tid}, 31;")
        cta = k.special("%ctaid.x")
        blk = block_indices(k, cta, ctx.tile, ctx.tile_axes()[:2])
        rb, cb = blk["a0_b"], blk["a5_b"]
        r0 = k.reg("r")
        k(f"mul.lo.u32 {r0}, {rb}, {BM};")
        c0 = k.reg("r")
        k(f"mul.lo.u32 {c0}, {cb}, {BD};")
        raw = k.reg("r")
        k(f"mov.u32 {raw}, __emmy_smem;")
        sm = k.reg("r")
        k(f"add.u32 {sm}, {raw}, 1023;")
        k(f"and.b32 {sm}, {sm}, -1024;")
        bsm = k.reg("r")                       # B region: after A and A_lo
        k(f"add.u32 {bsm}, {sm}, {2 * sa};")
        bar = k.reg("r")
        k(f"add.u32 {bar}, {sm}, {self.need - 1024 - 64};")
        tslot = k.reg("r")
        k(f"add.u32 {tslot}, {bar}, 16;")
        status = k.reg("rd")
        k(f"mov.u64 {status}, __emmy_status;")
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip = k.label("SKIP_INIT")
        k(f"@!{p0} bra {skip};")
        k(f"mbarrier.init.shared::cta.b64 [{bar}], 1;")
        k("fence.mbarrier_init.release.cluster;")
        k.mark(skip)
        pw0 = k.reg("p")
        k(f"setp.eq.u32 {pw0}, {warp}, 0;")
        skip2 = k.label("SKIP_ALLOC")
        k(f"@!{pw0} bra {skip2};")
        k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{tslot}], {self.ncols};")
        k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
        k.mark(skip2)
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
        k("tcgen05.fence::after_thread_sync;")
        tmem = k.reg("r")
        k(f"ld.shared.u32 {tmem}, [{tslot}];")
        teardown = k.label("TEARDOWN")
        hi = _desc_hi(16, 1024)
        ptrue = k.reg("p")
        k(f"setp.eq.u32 {ptrue}, 0, 0;")
        wait = GemmTemplate._wait
        st = Stager(k, tid, T, 4, True)
        nph = [0]                              # completions of the one barrier so far

        def mma_and_wait(first, n_cols, acc_col, nsteps):
            """Thread 0 issues one slab's 3xTF32 MMAs (A at sm, B at bsm, low
            parts after each) into TMEM column ``acc_col``; everyone waits."""
            k("fence.proxy.async.shared::cta;")
            k("bar.sync 0;")
            sk = k.label("NO_MMA")
            k(f"@!{p0} bra {sk};")
            k("tcgen05.fence::after_thread_sync;")
            da = GemmTemplate._desc(k, sm, hi)
            la = k.reg("r")
            k(f"add.u32 {la}, {sm}, {sa};")
            dla = GemmTemplate._desc(k, la, hi)
            db = GemmTemplate._desc(k, bsm, hi)
            lb = k.reg("r")
            k(f"add.u32 {lb}, {bsm}, {sb};")
            dlb = GemmTemplate._desc(k, lb, hi)
            idesc = k.reg("r")
            k(f"mov.u32 {idesc}, {idesc_mma(128, n_cols, False, True)};")
            dcol = k.reg("r")
            k(f"add.u32 {dcol}, {tmem}, {acc_col};")
            fst = True
            for s_ in range(nsteps):
                for x, y in ((dla, db), (da, dlb), (da, db)):
                    ax = k.reg("rd")
                    k(f"add.s64 {ax}, {x}, {2 * s_};")
                    by = k.reg("rd")
                    k(f"add.s64 {by}, {y}, {2 * s_};")
                    pa = first if fst else ptrue
                    fst = False
                    k(f"tcgen05.mma.cta_group::1.kind::tf32 [{dcol}], {ax}, {by}, {idesc}, {pa};")
            k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{bar}];")
            k.mark(sk)
            wait(k, bar, nph[0] & 1, status, 2, teardown)
            nph[0] += 1
            k("tcgen05.fence::after_thread_sync;")

        zero = k.reg("r")
        k(f"mov.u32 {zero}, 0;")
        # ---------------- S = Q kt (32 columns of d a slab) ----------------
        for s_ in range(-(-d // 32)):
            kbv = k.reg("r")
            k(f"mov.u32 {kbv}, {32 * s_};")
            ca = st.fetch("K", kbv, r0, BM, Sq, qb, d, d, d % 4 == 0)
            cbk = st.fetch("T", kbv, zero, S, S, kb_, S, d)
            st.put(ca, sm, sa)
            st.put(cbk, bsm, sb)
            first = k.reg("p")
            k(f"setp.ne.u32 {first}, {s_}, 0;")
            mma_and_wait(first, Sp, 0, -(-min(32, d - 32 * s_) // 8))
        # ---------------- the row max of the scaled scores ----------------
        warps = T // 32
        q4 = k.reg("r")
        k(f"and.b32 {q4}, {warp}, 3;")
        hasrows = k.reg("p")                   # this warp's TMEM lane quarter holds rows
        k(f"setp.lt.u32 {hasrows}, {q4}, {-(-BM // 32)};")
        if warps > 4:
            k(f"setp.lt.and.u32 {hasrows}, {warp}, 4, {hasrows};")
        lrow = k.reg("r")
        k(f"mad.lo.u32 {lrow}, {q4}, 32, {lane};")
        trow = k.reg("r")
        k(f"shl.b32 {trow}, {q4}, 21;")
        k(f"add.u32 {trow}, {trow}, {tmem};")
        c = k.reg("f")
        k(f"ld.global.nc.f32 {c}, [{sbuf}];")
        k(f"rcp.rn.f32 {c}, {c};")
        k(f"mul.rn.f32 {c}, {c}, 0f{_f32hex(LOG2E)};")
        m = k.reg("f")
        k(f"mov.f32 {m}, 0fFF800000;")
        lsum = k.reg("f")
        k(f"mov.f32 {lsum}, 0f00000000;")
        chunks16 = list(range(0, Sp, 16))
        norows = k.label("NO_ROWS_MAX")
        k(f"@!{hasrows} bra {norows};")
        for c16 in chunks16:
            regs = k.regs("r", 16)
            k(f"tcgen05.ld.sync.aligned.32x32b.x16.b32 {{{', '.join(regs)}}}, [{trow}+{c16}];")
            k("tcgen05.wait::ld.sync.aligned;")
            for e, r_ in enumerate(regs):
                if c16 + e >= S:
                    break
                x = k.reg("f")
                k(f"mul.rn.f32 {x}, {r_}, {c};")
                k(f"max.f32 {m}, {m}, {x};")
        k.mark(norows)
        # ---------------- O += P V, 32 keys a slab ----------------
        sk_rows = k.reg("p")                   # rows stored into the P operand
        k(f"setp.lt.and.u32 {sk_rows}, {lrow}, {-(-BM // 8) * 8}, {hasrows};")
        for t in range(-(-S // 32)):
            keys = min(32, S - 32 * t)
            nop = k.label("NO_P")
            k(f"@!{hasrows} bra {nop};")
            cols = [c16 for c16 in chunks16 if 32 * t <= c16 < 32 * t + 32]
            pv = []
            for c16 in cols:
                regs = k.regs("r", 16)
                k(f"tcgen05.ld.sync.aligned.32x32b.x16.b32 {{{', '.join(regs)}}}, [{trow}+{c16}];")
                pv.extend(regs)
            k("tcgen05.wait::ld.sync.aligned;")
            ps = []
            for e in range(32):
                p_ = k.reg("r")
                if e < keys:
                    x = k.reg("f")
                    k(f"mul.rn.f32 {x}, {pv[e]}, {c};")
                    k(f"sub.rn.f32 {x}, {x}, {m};")
                    k(f"ex2.approx.ftz.f32 {x}, {x};")
                    k(f"add.rn.f32 {lsum}, {lsum}, {x};")
                    k(f"mov.b32 {p_}, {x};")
                else:
                    k(f"mov.b32 {p_}, 0;")
                ps.append(p_)
            skst = k.label("NO_P_STORE")
            k(f"@!{sk_rows} bra {skst};")
            for ch in range(8):
                chr_ = k.reg("r")
                k(f"mov.u32 {chr_}, {ch};")
                st.store_chunk(sm, st.swz(lrow, chr_), ps[4 * ch:4 * ch + 4], sa)
            k.mark(skst)
            k.mark(nop)
            kbv = k.reg("r")
            k(f"mov.u32 {kbv}, {32 * t};")
            cv = st.fetch("T", kbv, c0, BD, dv, vb, dv, S)
            st.put(cv, bsm, sb)
            first = k.reg("p")
            k(f"setp.ne.u32 {first}, {t}, 0;")
            mma_and_wait(first, BDp, ocol, -(-keys // 8))
        # ---------------- O / l ----------------
        noep = k.label("NO_ROWS_OUT")
        k(f"@!{hasrows} bra {noep};")
        inv = k.reg("f")
        k(f"rcp.rn.f32 {inv}, {lsum};")
        grow = k.reg("r")
        k(f"add.u32 {grow}, {r0}, {lrow};")
        rok = k.reg("p")
        k(f"setp.lt.u32 {rok}, {lrow}, {BM};")
        orow = k.reg("rd")
        k(f"mul.wide.u32 {orow}, {grow}, {dv * 4};")
        k(f"add.s64 {orow}, {orow}, {ob};")
        for c8 in range(0, BDp, 8):
            regs = k.regs("r", 8)
            k(f"tcgen05.ld.sync.aligned.32x32b.x8.b32 {{{', '.join(regs)}}}, "
              f"[{trow}+{ocol + c8}];")
            k("tcgen05.wait::ld.sync.aligned;")
            for e in range(8):
                if c8 + e >= BD:
                    break
                y = k.reg("f")
                k(f"mul.rn.f32 {y}, {regs[e]}, {inv};")
                gc = k.reg("r")
                k(f"add.u32 {gc}, {c0}, {c8 + e};")
                a = k.reg("rd")
                k(f"mul.wide.u32 {a}, {gc}, 4;")
                k(f"add.s64 {a}, {a}, {orow};")
                k(f"@{rok} st.global.f32 [{a}], {y};")
        k.mark(noep)
        # ---------------- teardown ----------------
        k.mark(teardown)
        k("tcgen05.fence::before_thread_sync;")
        k("barrier.sync 0;")
        end = k.label("END")
        k(f"@!{pw0} bra {end};")
        k("bar.warp.sync 0xffffffff;")
        k("tcgen05.fence::after_thread_sync;")
        k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {self.ncols};")
        k.mark(end)
        k("ret;")
        return k.render()

"""Attention template: ``O = softmax(Q K^T * s) V`` as a flash-attention kernel
on the 5th-generation tensor cores.

Matches Emmy's attention schedule (reference ``problems/a01_attention``,
``a02_attention_128``: per key ``a1``, a q.k dot-product ``Loop`` per output
row, the online-softmax ``Assign``/``Accum`` chain with the running max
(``acc1``), the running sum (``acc3``) and the weighted sum of V (``acc5``),
then ``reciprocal`` + ``multiply``), here with leading batch/head axes, bf16
Q/K/V [B,H,S,D] and an f32 output.  The reference lowers each thread's
micro-tile to scalar FFMAs that recompute the scores per output column
(``compile.py:1882-1928``).  This template keeps the IR's CTA -> (batch,
head, 128 query rows) assignment and computes the tile as:

* TMA loads the CTA's Q tile once and K and V tiles of 128 keys into two
  separate rings (3 + 2 stages at D=128, 4 + 4 at D=64; 128-byte swizzle;
  no multicast), each fed by its own producer thread, so a K tile is reused
  as soon as its Q.K^T has run and the loads stay ahead of the MMAs;
* one thread issues ``S_j = Q K_j^T`` (``tcgen05.mma kind::f16``, M=N=128)
  into one of two TMEM score buffers, and ``O += P_{j-1} V_{j-1}`` with P read
  from TMEM (the ``[a-tmem]`` form) and V as an MN-major shared operand, so
  the scores of block j+1 overlap the softmax of block j;
* eight softmax warps, two threads per query row (the row is the thread's
  TMEM lane; each thread owns half of the 128 score columns and half of the
  D output columns): half-row maxima exchanged through shared memory under a
  64-arrival mbarrier, ``p = 2^(s*c - m)`` (c = s*log2 e), P written back
  over S as packed bf16 pairs, partial row sums; the exponent base m moves
  only when the row max grows by more than 2^8, and only then is the running
  O row rescaled in TMEM by ``2^(m_old - m_new)`` (the same base is used for
  the final 1/l, so this is exact);
* after the last block the two half sums are added and each thread scales
  its half of the O row by 1/l and stores it.

The arithmetic is the IR's: the same online-softmax recurrence (max, the
exp rescale factor of the previous state, sum, weighted sum), evaluated per
128-key block instead of per key.  Every mbarrier wait is bounded by
``%globaltimer`` (2 s) and reports through ``__emmy_status``.
"""
from __future__ import annotations

from ..analysis import NotAffine, affine, kind, walk
from ..ptx import Kernel
from .common import TemplateMismatch
from .gemm import GemmTemplate, _desc_hi, idesc_mma

LOG2E = 1.4426950408889634


class AttentionTemplate:
    name = "attention"

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "AttentionTemplate":
        tile = ctx.tile
        if tile is None:
            raise TemplateMismatch("no single top-level Tile")
        axes = ctx.tile_axes()
        names = [a for a, _ in axes]
        if names != ["ab", "ah", "a0_b", "a5_b", "a0_u", "a5_u"]:
            raise TemplateMismatch("not a batched attention tile")
        ext = dict(axes)
        body = list(tile.body)
        keyloops = [s for s in body if kind(s) == "Loop"]
        if len(keyloops) != 1:
            raise TemplateMismatch("expected one key loop")
        kl = keyloops[0]
        key = kl.axis.name
        bufs = ctx.bufs
        # the scale: v = reciprocal(load c[0]) multiplies the dot product
        scale_buf = None
        for s in body:
            if kind(s) == "Load" and s is not kl:
                try:
                    if all(affine(i).is_const() for i in s.index) and bufs.size(s.input) == 1:
                        scale_buf = s.input
                except NotAffine:
                    pass
        if scale_buf is None:
            raise TemplateMismatch("no scale constant")
        q = k_ = v = None
        ops = set()
        for s in walk(kl.body):
            kd = kind(s)
            if kd == "Loop":
                for t in s.body:
                    if kind(t) == "Load":
                        fv = set().union(*(i.free_vars() for i in t.index))
                        if key in fv:
                            k_ = k_ or t.input
                            if t.input != k_:
                                raise TemplateMismatch("two key operands")
                        elif "a0_u" in fv:
                            q = q or t.input
                            if t.input != q:
                                raise TemplateMismatch("two query operands")
            elif kd == "Load":
                fv = set().union(*(i.free_vars() for i in s.index))
                if key in fv and "a5_u" in fv and s.input not in (q, k_):
                    v = v or s.input
            elif kd in ("Assign", "Accum"):
                ops.add(s.op.name)
        if not (q and k_ and v) or len({q, k_, v}) != 3:
            raise TemplateMismatch("q/k/v operands")
        if not {"exp", "maximum", "multiply", "add", "subtract"} <= ops or \
                ops - {"exp", "maximum", "multiply", "add", "subtract", "copy"}:
            raise TemplateMismatch(f"softmax chain ops {sorted(ops)}")
        writes = [s for s in body if kind(s) == "Write"]
        outs = {w.output for w in writes}
        if len(outs) != 1 or any(w.atomic for w in writes):
            raise TemplateMismatch("output")
        out = outs.pop()
        shp = bufs.shapes[q]
        if len(shp) != 4 or bufs.shapes[k_] != shp or bufs.shapes[v] != shp or \
                bufs.shapes[out] != shp:
            raise TemplateMismatch("q/k/v/out shapes")
        if {bufs.dtypes[q], bufs.dtypes[k_], bufs.dtypes[v]} != {"bf16"} or \
                bufs.dtypes[out] != "f32":
            raise TemplateMismatch("dtypes (bf16 in, f32 out)")
        B, H, S, D = shp
        BM = None
        for w in writes:
            r = affine(w.index[2])
            BM = r.coef("a0_b")
        if BM != 128 or ext["a0_b"] * 128 != S or ext["a5_b"] != 1 or D not in (64, 128) or \
                S % 128 or ext["ab"] != B or ext["ah"] != H:
            raise TemplateMismatch("tile geometry")
        if ctx.block != (512, 1, 1) or ctx.grid[0] * ctx.grid[1] * ctx.grid[2] != B * H * S // 128:
            raise TemplateMismatch("launch geometry")
        self = cls()
        self.ctx, self.q, self.k, self.v, self.out, self.scale_buf = ctx, q, k_, v, out, scale_buf
        self.B, self.H, self.S, self.D = B, H, S, D
        self.tile_bytes = TB = 128 * D * 2
        # Q tile + K ring + V ring, sized from the launch's shared memory
        avail = min(ctx.smem_bytes, 227 * 1024) - 1024 - 512 - 3072 - TB
        n = min(8, avail // TB)
        if n < 4:
            raise TemplateMismatch("meta smem_bytes too small for 2+2 K/V stages")
        self.SK, self.SV = (n + 1) // 2, n // 2
        return self

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        ctx = self.ctx
        D, S = self.D, self.S
        NB = S // 128                      # key blocks
        QB = S // 128                      # query blocks per head
        TB = self.tile_bytes               # one 128 x D bf16 tile
        NBX = D // 64                      # 64-column boxes per tile
        params = ctx.params() + [("tmapQ", ".align 64 .b8", "[128]"),
                                 ("tmapK", ".align 64 .b8", "[128]"),
                                 ("tmapV", ".align 64 .b8", "[128]")]
        k = Kernel(ctx.entry, params)
        k.maxntid = (512, 1, 1)
        k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
        k.decl(".global .align 4 .u32 __emmy_status;")
        rows = self.B * self.H * S
        for nm, buf in (("tmapQ", self.q), ("tmapK", self.k), ("tmapV", self.v)):
            k.directive(f"tmap {nm} buf={buf} dtype=9 dims={D},{rows} strides={D * 2} "
                        f"box=64,128 swizzle=3")
        k.comment(f"emmy-b200 template: tcgen05 flash attention B={self.B} H={self.H} S={S} D={D}")
        obase = k.param_ptr(self.out)
        sbuf = k.param_ptr(self.scale_buf)
        tq, tk, tv = (k.reg("rd") for _ in range(3))
        for r, nm in ((tq, "tmapQ"), (tk, "tmapK"), (tv, "tmapV")):
            k(f"mov.u64 {r}, param_{nm};")
            k(f"cvta.param.u64 {r}, {r};")
        tid = k.special("%tid.x")
        warp = k.reg("r")
        k(f"shr.u32 {warp}, {tid}, 5;")
        lane = k.reg("r")
        k(f"and.b32 {lane}, {tid}, 31;")
        cta = k.special("%ctaid.x")
        bh = k.reg("r")
        k(f"div.u32 {bh}, {cta}, {QB};")
        qb = k.reg("r")
        k(f"rem.u32 {qb}, {cta}, {QB};")
        krow0 = k.reg("r")
        k(f"mul.lo.u32 {krow0}, {bh}, {S};")
        qrow0 = k.reg("r")
        k(f"mad.lo.u32 {qrow0}, {qb}, 128, {krow0};")
        SK, SV = self.SK, self.SV
        # shared memory: Q | K ring (SK tiles) | V ring (SV tiles) | barriers |
        # tmem slot | row exchange
        raw = k.reg("r")
        k(f"mov.u32 {raw}, __emmy_smem;")
        qs = k.reg("r")
        k(f"add.u32 {qs}, {raw}, 1023;")
        k(f"and.b32 {qs}, {qs}, -1024;")
        kring = k.reg("r")
        k(f"add.u32 {kring}, {qs}, {TB};")
        vring = k.reg("r")
        k(f"add.u32 {vring}, {kring}, {SK * TB};")
        bars = k.reg("r")
        k(f"add.u32 {bars}, {vring}, {SV * TB};")
        # barrier slots
        Q_FULL = 0
        K_FULL, K_EMPTY = 1, 1 + SK
        V_FULL, V_EMPTY = 1 + 2 * SK, 1 + 2 * SK + SV
        S_FULL = 1 + 2 * SK + 2 * SV
        P_READY = S_FULL + 2
        O_DONE = P_READY + 2
        FINAL = O_DONE + 1
        XBAR = FINAL + 1          # xbar[q]: the two warps of row quarter q (64 arrivals)
        NSLOT = XBAR + 4
        tslot = k.reg("r")
        k(f"add.u32 {tslot}, {bars}, {NSLOT * 8};")
        # row-max / row-sum exchange between the two threads of a row:
        # xch[parity][half][row] f32 at bars + 512, the final sums at +2048
        xch = k.reg("r")
        k(f"add.u32 {xch}, {bars}, 512;")
        status = k.reg("rd")
        k(f"mov.u64 {status}, __emmy_status;")
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip = k.label("SKIP_INIT")
        k(f"@!{p0} bra {skip};")
        for slot in range(NSLOT):
            cnt = 256 if slot in (P_READY, P_READY + 1) else 64 if slot >= XBAR else 1
            k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * slot}], {cnt};")
        k("fence.mbarrier_init.release.cluster;")
        for r in (tq, tk, tv):
            k(f"prefetch.tensormap [{r}];")
        k.mark(skip)
        pw1 = k.reg("p")
        k(f"setp.eq.u32 {pw1}, {warp}, 1;")
        skip2 = k.label("SKIP_ALLOC")
        k(f"@!{pw1} bra {skip2};")
        k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{tslot}], 512;")
        k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
        k.mark(skip2)
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
        k("tcgen05.fence::after_thread_sync;")
        tmem = k.reg("r")
        k(f"ld.shared.u32 {tmem}, [{tslot}];")
        teardown = k.label("TEARDOWN")
        pl0 = k.reg("p")
        k(f"setp.eq.u32 {pl0}, {lane}, 0;")
        wait = GemmTemplate._wait

        def bar(slot, idx=None):
            """Address of barrier ``slot`` (+ a 0/1 register index)."""
            r = k.reg("r")
            if idx is None:
                k(f"add.u32 {r}, {bars}, {8 * slot};")
            else:
                k(f"mad.lo.u32 {r}, {idx}, 8, {bars};")
                k(f"add.u32 {r}, {r}, {8 * slot};")
            return r

        j = k.reg("r")
        b = k.reg("r")      # j % 2  (ring stage and score buffer)
        ph = k.reg("r")     # (j / 2) % 2

        def split(jreg):
            k(f"and.b32 {b}, {jreg}, 1;")
            k(f"shr.u32 {ph}, {jreg}, 1;")
            k(f"and.b32 {ph}, {ph}, 1;")

        def ring_slot(jreg, depth):
            """(stage, phase) of block j in a ring of ``depth`` stages."""
            st_ = k.reg("r")
            k(f"rem.u32 {st_}, {jreg}, {depth};")
            ph_ = k.reg("r")
            k(f"div.u32 {ph_}, {jreg}, {depth};")
            k(f"and.b32 {ph_}, {ph_}, 1;")
            return st_, ph_

        def producer(which, warp_id, tmap, ring, depth, full, empty, load_q):
            pp = k.reg("p")
            k(f"setp.eq.u32 {pp}, {warp}, {warp_id};")
            k(f"and.pred {pp}, {pp}, {pl0};")
            end_p = k.label(f"END_{which}")
            k(f"@!{pp} bra {end_p};")
            if load_q:
                qf = bar(Q_FULL)
                k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{qf}], {TB};")
                for i in range(NBX):
                    k(f"cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
                      f"[{qs}+{i * 16384}], [{tq}, {{{64 * i}, {qrow0}}}], [{qf}];")
            k(f"mov.u32 {j}, 0;")
            top = k.label(f"PROD_{which}")
            k.mark(top)
            st_, ph_ = ring_slot(j, depth)
            par = k.reg("r")
            k(f"xor.b32 {par}, {ph_}, 1;")
            wait(k, bar(empty, st_), par, status, 1, end_p)
            kr = k.reg("r")
            k(f"mad.lo.u32 {kr}, {j}, 128, {krow0};")
            dst = k.reg("r")
            k(f"mad.lo.u32 {dst}, {st_}, {TB}, {ring};")
            fb = bar(full, st_)
            k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {TB};")
            for i in range(NBX):
                k(f"cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
                  f"[{dst}+{i * 16384}], [{tmap}, {{{64 * i}, {kr}}}], [{fb}];")
            k(f"add.u32 {j}, {j}, 1;")
            pl = k.reg("p")
            k(f"setp.lt.u32 {pl}, {j}, {NB};")
            k(f"@{pl} bra {top};")
            k.mark(end_p)

        # ---------------- producers: K (and Q) on warp 0, V on warp 2 ----------------
        producer("K", 0, tk, kring, SK, K_FULL, K_EMPTY, True)
        producer("V", 2, tv, vring, SV, V_FULL, V_EMPTY, False)

        # ---------------- MMA issuer: warp 1 lane 0 ----------------
        pm = k.reg("p")
        k(f"setp.eq.u32 {pm}, {warp}, 1;")
        k(f"and.pred {pm}, {pm}, {pl0};")
        end_mma = k.label("END_MMA")
        k(f"@!{pm} bra {end_mma};")
        iqk = k.reg("r")
        k(f"mov.u32 {iqk}, {idesc_mma(128, 128, False)};")
        ipv = k.reg("r")
        k(f"mov.u32 {ipv}, {idesc_mma(128, D, True)};")
        hiK = _desc_hi(16, 1024)
        hiV = _desc_hi(16384, 1024)
        ptrue = k.reg("p")
        k(f"setp.eq.u32 {ptrue}, 0, 0;")
        zero = k.reg("r")
        k(f"mov.u32 {zero}, 0;")
        wait(k, bar(Q_FULL), zero, status, 2, end_mma)
        dq = GemmTemplate._desc(k, qs, hiK)
        o_tm = k.reg("r")
        k(f"add.u32 {o_tm}, {tmem}, 256;")

        def issue_qk(jreg):
            kst, kph = ring_slot(jreg, SK)
            wait(k, bar(K_FULL, kst), kph, status, 2, end_mma)
            k("tcgen05.fence::after_thread_sync;")
            kad = k.reg("r")
            k(f"mad.lo.u32 {kad}, {kst}, {TB}, {kring};")
            dk = GemmTemplate._desc(k, kad, hiK)
            sb = k.reg("r")
            k(f"and.b32 {sb}, {jreg}, 1;")
            s_tm = k.reg("r")
            k(f"mad.lo.u32 {s_tm}, {sb}, 128, {tmem};")
            pfirst = k.reg("p")
            k(f"setp.ne.u32 {pfirst}, 0, 0;")       # the first MMA overwrites S
            for kk in range(D // 16):
                off = (kk % 4) * 2 + (kk // 4) * 1024
                a = k.reg("rd")
                k(f"add.s64 {a}, {dq}, {off};")
                bd = k.reg("rd")
                k(f"add.s64 {bd}, {dk}, {off};")
                k(f"tcgen05.mma.cta_group::1.kind::f16 [{s_tm}], {a}, {bd}, {iqk}, "
                  f"{pfirst if kk == 0 else ptrue};")
            k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar(S_FULL, sb)}];")
            k.comment(f"@trace 0 {jreg}")
            k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar(K_EMPTY, kst)}];")

        def issue_pv(ireg, first_pred):
            split(ireg)
            wait(k, bar(P_READY, b), ph, status, 2, end_mma)
            k.comment(f"@trace 1 {ireg}")
            k("tcgen05.fence::after_thread_sync;")
            vst, vph = ring_slot(ireg, SV)
            wait(k, bar(V_FULL, vst), vph, status, 2, end_mma)
            vad = k.reg("r")
            k(f"mad.lo.u32 {vad}, {vst}, {TB}, {vring};")
            dv = GemmTemplate._desc(k, vad, hiV)
            p_tm = k.reg("r")
            k(f"mad.lo.u32 {p_tm}, {b}, 128, {tmem};")
            for kk in range(8):                     # 128 keys, K=16 per MMA
                a = k.reg("r")
                k(f"add.u32 {a}, {p_tm}, {8 * kk};")   # 16 bf16 = 8 TMEM columns
                bd = k.reg("rd")
                k(f"add.s64 {bd}, {dv}, {kk * 128};")  # +16 key rows * 128 B
                k(f"tcgen05.mma.cta_group::1.kind::f16 [{o_tm}], [{a}], {bd}, {ipv}, "
                  f"{first_pred if kk == 0 else ptrue};")
            k.comment(f"@trace 2 {ireg}")
            k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar(O_DONE)}];")
            k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar(V_EMPTY, vst)}];")

        k(f"mov.u32 {j}, 0;")
        issue_qk(j)
        k(f"mov.u32 {j}, 1;")
        jm = k.reg("r")
        pacc = k.reg("p")
        if NB > 1:
            top2 = k.label("MMA")
            k.mark(top2)
            issue_qk(j)
            k(f"sub.u32 {jm}, {j}, 1;")
            k(f"setp.ne.u32 {pacc}, {jm}, 0;")
            issue_pv(jm, pacc)
            k(f"add.u32 {j}, {j}, 1;")
            pl2 = k.reg("p")
            k(f"setp.lt.u32 {pl2}, {j}, {NB};")
            k(f"@{pl2} bra {top2};")
        k(f"mov.u32 {jm}, {NB - 1};")
        k(f"setp.ne.u32 {pacc}, {jm}, 0;")
        issue_pv(jm, pacc)
        k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
          f"[{bar(FINAL)}];")
        k.mark(end_mma)

        # ------------- softmax warps 4-11: two threads per query row -------------
        # warp w: rows 32*(w%4) + lane (its TMEM lanes), half h = (w-4)/4 of the
        # 128 score columns and of the D output columns
        psm = k.reg("p")
        k(f"setp.ge.u32 {psm}, {warp}, 4;")
        psm2 = k.reg("p")
        k(f"setp.lt.u32 {psm2}, {warp}, 12;")
        k(f"and.pred {psm}, {psm}, {psm2};")
        end_sm = k.label("END_SM")
        k(f"@!{psm} bra {end_sm};")
        q4 = k.reg("r")
        k(f"and.b32 {q4}, {warp}, 3;")
        hh = k.reg("r")
        k(f"sub.u32 {hh}, {warp}, 4;")
        k(f"shr.u32 {hh}, {hh}, 2;")
        row = k.reg("r")
        k(f"mad.lo.u32 {row}, {q4}, 32, {lane};")
        trow = k.reg("r")
        k(f"shl.b32 {trow}, {q4}, 21;")            # TMEM lane field (32*q4) << 16
        k(f"add.u32 {trow}, {trow}, {tmem};")
        scol = k.reg("r")
        k(f"shl.b32 {scol}, {hh}, 6;")             # 64*h score columns
        pcol = k.reg("r")
        k(f"shl.b32 {pcol}, {hh}, 5;")             # 32*h packed P columns
        ocol = k.reg("r")
        k(f"mul.lo.u32 {ocol}, {hh}, {D // 2};")
        k(f"add.u32 {ocol}, {ocol}, 256;")
        otm = k.reg("r")
        k(f"add.u32 {otm}, {trow}, {ocol};")
        xb = k.reg("r")                            # exchange mbarrier of this row pair
        k(f"mad.lo.u32 {xb}, {q4}, 8, {bars};")
        k(f"add.u32 {xb}, {xb}, {8 * XBAR};")
        mine = k.reg("r")                          # &xch[0][h][row]
        k(f"mad.lo.u32 {mine}, {hh}, 512, {xch};")
        k(f"mad.lo.u32 {mine}, {row}, 4, {mine};")
        other = k.reg("r")                         # &xch[0][1-h][row]
        k(f"xor.b32 {other}, {hh}, 1;")
        k(f"mad.lo.u32 {other}, {other}, 512, {xch};")
        k(f"mad.lo.u32 {other}, {row}, 4, {other};")
        sc = k.reg("f")
        k(f"ld.global.nc.f32 {sc}, [{sbuf}];")
        k(f"rcp.rn.f32 {sc}, {sc};")
        k(f"mul.rn.f32 {sc}, {sc}, 0f{_f32hex(LOG2E)};")     # c = s * log2(e)
        m = k.reg("f")                             # max used for the exponents
        k(f"mov.f32 {m}, 0fFF800000;")
        lsum = k.reg("f")
        k(f"mov.f32 {lsum}, 0f00000000;")
        k(f"mov.u32 {j}, 0;")
        top3 = k.label("SMX")
        k.mark(top3)
        split(j)
        wait(k, bar(S_FULL, b), ph, status, 3, teardown)
        k.comment(f"@trace 3 {j}")
        k("tcgen05.fence::after_thread_sync;")
        srow = k.reg("r")
        k(f"mad.lo.u32 {srow}, {b}, 128, {trow};")
        sa = k.reg("r")
        k(f"add.u32 {sa}, {srow}, {scol};")
        sv = k.regs("r", 64)
        for c2 in range(2):
            k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(sv[32 * c2:32 * c2 + 32])}}}, "
              f"[{sa}+{32 * c2}];")
        k("tcgen05.wait::ld.sync.aligned;")
        mx = [k.reg("f") for _ in range(8)]
        for i in range(8):
            k(f"max.f32 {mx[i]}, {sv[i]}, {sv[i + 8]};")
        for i in range(16, 64):
            k(f"max.f32 {mx[i % 8]}, {mx[i % 8]}, {sv[i]};")
        for w in (4, 2, 1):
            for i in range(w):
                k(f"max.f32 {mx[i]}, {mx[i]}, {mx[i + w]};")
        # exchange the half-row maxima (buffer by iteration parity)
        par2 = k.reg("r")
        k(f"and.b32 {par2}, {j}, 1;")
        po = k.reg("r")
        k(f"shl.b32 {po}, {par2}, 10;")
        wa = k.reg("r")
        k(f"add.u32 {wa}, {mine}, {po};")
        k(f"st.shared.f32 [{wa}], {mx[0]};")
        k(f"mbarrier.arrive.shared::cta.b64 _, [{xb}];")
        wait(k, xb, par2, status, 5, teardown)
        ra = k.reg("r")
        k(f"add.u32 {ra}, {other}, {po};")
        om = k.reg("f")
        k(f"ld.shared.f32 {om}, [{ra}];")
        k(f"max.f32 {mx[0]}, {mx[0]}, {om};")
        # lazy rescaling: move the exponent base only when the row max grew by
        # more than 2^8 (p stays <= 256); the final 1/l uses the same base
        cand = k.reg("f")
        k(f"mul.rn.f32 {cand}, {mx[0]}, {sc};")
        thr = k.reg("f")
        k(f"add.rn.f32 {thr}, {m}, 0f41000000;")         # m + 8
        need = k.reg("p")
        k(f"setp.gt.f32 {need}, {cand}, {thr};")
        meff = k.reg("f")
        k(f"selp.f32 {meff}, {cand}, {m}, {need};")
        alpha = k.reg("f")
        dlt = k.reg("f")
        k(f"sub.rn.f32 {dlt}, {m}, {meff};")
        k(f"ex2.approx.ftz.f32 {alpha}, {dlt};")
        k(f"@!{need} mov.f32 {alpha}, 0f3F800000;")
        negm = k.reg("f")
        k(f"neg.f32 {negm}, {meff};")
        ps = [k.reg("f") for _ in range(8)]
        packed = k.regs("r", 32)
        for i in range(0, 64, 2):
            e2 = []
            for ii in (i, i + 1):
                t = k.reg("f")
                k(f"fma.rn.f32 {t}, {sv[ii]}, {sc}, {negm};")
                e = k.reg("f")
                k(f"ex2.approx.ftz.f32 {e}, {t};")
                if ii < 8:
                    k(f"mov.f32 {ps[ii]}, {e};")
                else:
                    k(f"add.rn.f32 {ps[ii % 8]}, {ps[ii % 8]}, {e};")
                e2.append(e)
            k(f"cvt.rn.bf16x2.f32 {packed[i // 2]}, {e2[1]}, {e2[0]};")
        pa = k.reg("r")
        k(f"add.u32 {pa}, {srow}, {pcol};")
        k(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{pa}], {{{', '.join(packed)}}};")
        k.comment(f"@trace 4 {j}")
        for w in (4, 2, 1):
            for i in range(w):
                k(f"add.rn.f32 {ps[i]}, {ps[i]}, {ps[i + w]};")
        k(f"fma.rn.f32 {lsum}, {lsum}, {alpha}, {ps[0]};")
        # rescale this warp's half of the running O rows if any of its rows
        # moved (warp-uniform), after the previous P.V has landed
        skip_rs = k.label("NO_RESCALE")
        pj0 = k.reg("p")
        k(f"setp.eq.u32 {pj0}, {j}, 0;")
        k(f"@{pj0} bra {skip_rs};")
        anyw = k.reg("p")
        k(f"vote.sync.any.pred {anyw}, {need}, 0xffffffff;")
        k(f"@!{anyw} bra {skip_rs};")
        jp = k.reg("r")
        k(f"sub.u32 {jp}, {j}, 1;")
        k(f"and.b32 {jp}, {jp}, 1;")
        wait(k, bar(O_DONE), jp, status, 3, teardown)
        k("tcgen05.fence::after_thread_sync;")
        half = D // 2
        ov = k.regs("r", half)
        for c in range(half // 32):
            k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov[32 * c:32 * c + 32])}}}, "
              f"[{otm}+{32 * c}];")
        k("tcgen05.wait::ld.sync.aligned;")
        for r in ov:
            k(f"mul.rn.f32 {r}, {r}, {alpha};")
        for c in range(half // 32):
            k(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{otm}+{32 * c}], "
              f"{{{', '.join(ov[32 * c:32 * c + 32])}}};")
        k.mark(skip_rs)
        k("tcgen05.wait::st.sync.aligned;")
        k("tcgen05.fence::before_thread_sync;")
        k(f"mbarrier.arrive.shared::cta.b64 _, [{bar(P_READY, b)}];")
        k.comment(f"@trace 5 {j}")
        k(f"mov.f32 {m}, {meff};")
        k(f"add.u32 {j}, {j}, 1;")
        pl3 = k.reg("p")
        k(f"setp.lt.u32 {pl3}, {j}, {NB};")
        k(f"@{pl3} bra {top3};")
        # epilogue: row sum of both halves, O half-row * (1 / l) -> global
        k(f"st.shared.f32 [{mine}+2048], {lsum};")
        k(f"mbarrier.arrive.shared::cta.b64 _, [{xb}];")
        k(f"mov.u32 {par2}, {NB & 1};")
        wait(k, xb, par2, status, 5, teardown)
        ol = k.reg("f")
        k(f"ld.shared.f32 {ol}, [{other}+2048];")
        k(f"add.rn.f32 {lsum}, {lsum}, {ol};")
        wait(k, bar(FINAL), self._zero(k), status, 3, teardown)
        k("tcgen05.fence::after_thread_sync;")
        inv = k.reg("f")
        k(f"rcp.rn.f32 {inv}, {lsum};")
        orow = k.reg("r")
        k(f"add.u32 {orow}, {qrow0}, {row};")
        oa = k.reg("rd")
        k(f"mul.wide.u32 {oa}, {orow}, {D * 4};")
        k(f"add.s64 {oa}, {oa}, {obase};")
        hoff = k.reg("rd")
        k(f"mul.wide.u32 {hoff}, {hh}, {half * 4};")
        k(f"add.s64 {oa}, {oa}, {hoff};")
        for c in range(half // 32):
            regs = k.regs("r", 32)
            k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{otm}+{32 * c}];")
            k("tcgen05.wait::ld.sync.aligned;")
            for r in regs:
                k(f"mul.rn.f32 {r}, {r}, {inv};")
            for v8 in range(4):
                k(f"st.global.v8.b32 [{oa}+{128 * c + 32 * v8}], "
                  f"{{{', '.join(regs[8 * v8:8 * v8 + 8])}}};")
        k.mark(end_sm)

        # ---------------- teardown ----------------
        k.mark(teardown)
        k("tcgen05.fence::before_thread_sync;")
        k("barrier.sync 0;")
        end = k.label("END")
        k(f"@!{pw1} bra {end};")
        k("bar.warp.sync 0xffffffff;")
        k("tcgen05.fence::after_thread_sync;")
        k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, 512;")
        k.mark(end)
        k("ret;")
        return k.render()

    @staticmethod
    def _zero(k):
        r = k.reg("r")
        k(f"mov.u32 {r}, 0;")
        return r


def _f32hex(v: float) -> str:
    import struct
    return "%08X" % struct.unpack("<I", struct.pack("<f", float(v)))[0]

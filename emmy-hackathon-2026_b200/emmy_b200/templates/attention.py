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
head, BM query rows) assignment, BM = 128 * NT with NT = 1 or 2 query tiles
of 128 rows, and computes the CTA's rows as:

* TMA loads the NT Q tiles once and K and V tiles of 128 keys into two
  separate rings (3 + 2 stages at D=128, 4 + 4 at D=64; 128-byte swizzle;
  one copy per CTA), each fed by its own producer thread;
* one thread issues, per key block j and query tile t, ``O_t += P_t V_j``
  (P read from TMEM, the ``[a-tmem]`` form; V an MN-major shared operand)
  followed by ``S_t = Q_t K_{j+1}^T`` (M=N=128) into the tile's TMEM score
  buffer.  With two tiles the tensor pipe works on one tile while the other
  tile's softmax runs (ping-pong), so neither waits for the other;
* four softmax warps per tile, one thread per query row (the row is the
  thread's TMEM lane): the row max over the 128 scores (read in two halves),
  ``p = 2^(s*c - m)`` (c = s*log2 e) written back over S as packed bf16
  pairs, the row sum; the exponent base m moves only when the row max grows
  by more than 2^8, and only then is the running O row rescaled in TMEM by
  ``2^(m_old - m_new)`` (the same base is used for the final 1/l, so this is
  exact).  O_t is idle at that point: the previous ``P V`` of the tile is
  ordered before the ``Q K^T`` whose completion released the scores;
* after the last block each thread scales its O row by 1/l and stores it.

TMEM: S_t at columns 128 t, O_t at 256 + D t (512 columns allocated).  The
arithmetic is the IR's: the same online-softmax recurrence (max, the exp
rescale factor of the previous state, sum, weighted sum), evaluated per
128-key block instead of per key.  Every mbarrier wait is bounded by
``%globaltimer`` (2 s) and reports through ``__emmy_status``.
"""
from __future__ import annotations

import struct

from ..analysis import NotAffine, affine, kind, walk
from ..ptx import Kernel
from .common import TemplateMismatch
from .gemm import GemmTemplate, _desc_hi, idesc_mma

LOG2E = 1.4426950408889634
SMEM_MAX = 227 * 1024
# 2^f on [-0.5, 0.5]: degree-3 polynomial minimising the maximum relative
# error (linear-programming fit on 4001 points; 7.5e-5), f32 coefficients
EXP2_POLY = (0.9999280571937561, 0.6932608485221863, 0.24261115491390228, 0.05517221987247467)

# warp roles (512 threads): softmax warps 0..4*NT-1, then these
MMA_WARP, PROD_K_WARP, PROD_V_WARP = 8, 9, 10
# registers per thread: at launch, and after setmaxnreg for the softmax
# warpgroups and for the rest (2 x 128 x 200 + 2 x 128 x 56 = 512 x 128)
LAUNCH_REGS, SOFT_REGS, ROLE_REGS = 128, 200, 56


class AttentionTemplate:
    name = "attention"
    # column pairs per 16 whose exp2 runs on the FMA pipe instead of the
    # MUFU, by head dim (measured: a polynomial pair costs more issue and
    # FMA-pipe time than two MUFU ex2, so only the MUFU-bound D=64 gains;
    # there 3 of 16 beat 2, 4, 5 and 6)
    POLY = {64: 3, 128: 0}
    # P pass software pipeline: the scale of pair s+LEAD and the sum/pack of
    # pair s-LAG issue around the exponentials of pair s (measured: depth
    # 1/2, 1/4 and 2/6 time the same)
    PIPE = (1, 2)
    # wait for the next K block at the top of the MMA thread's block loop
    EARLY_K = True
    # head dims whose P gets TMEM columns of its own (S_t at 128 t, P_t at
    # 256 + 64 t, O_t at 384 + D t: 512 columns at D = 64 with two tiles).
    # The tiles then share their barriers and the MMA thread commits twice
    # per block (a commit costs the issuing thread about 100 cycles): at
    # D = 64 712 TFLOP/s against 703 with P over S (with per-tile barriers
    # and six commits per block the same split measured 679).
    # Then each tile's scores are released as soon as the softmax warps hold
    # them in registers, the next Q K^T runs while the softmax works, and the
    # softmax of block j+1 starts right after that of block j; P V of block
    # j overlaps it.  At D = 128 the columns do not fit: P overwrites S and
    # the tile's next Q K^T waits for its P V.
    SPLIT_P = {64: True, 128: False}
    # head dims whose CTAs run in pairs (a cluster of 2 over neighbouring
    # 256-row query blocks of one (batch, head)): the leader's one thread
    # issues tcgen05.mma.cta_group::2 (M = 256: each CTA's 128 rows of a tile
    # in its own TMEM), each CTA loads half of every K block (64 keys) and
    # half of every V block (D/2 columns), so per SM the MMA issue and the
    # K/V shared-memory traffic halve.  Correct, and slower at D = 128 (933
    # against 1178 TFLOP/s): a trace shows each tile's MMA chain shorter
    # but the two tiles' softmax passes in phase, contending for the MUFU
    # (3,200 cycles a pass instead of 1,750), a 4,570-cycle block period
    PAIR = {64: False, 128: False}

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "AttentionTemplate":
        from .gemm_small import meta_only
        if meta_only():
            raise TemplateMismatch("meta-only launch requested (EMMY_META_ONLY): no tensor maps")
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
        if BM not in (128, 256) or ext["a0_b"] * BM != S or ext["a5_b"] != 1 or \
                D not in (64, 128) or S % 128 or ext["ab"] != B or ext["ah"] != H:
            raise TemplateMismatch("tile geometry")
        if ctx.block != (512, 1, 1) or ctx.grid[0] * ctx.grid[1] * ctx.grid[2] != B * H * S // BM:
            raise TemplateMismatch("launch geometry")
        self = cls()
        self.ctx, self.q, self.k, self.v, self.out, self.scale_buf = ctx, q, k_, v, out, scale_buf
        self.B, self.H, self.S, self.D = B, H, S, D
        self.NT = BM // 128
        self.tile_bytes = TB = 128 * D * 2
        # Q tiles + K ring + V ring, sized from the launch's shared memory
        avail = min(ctx.smem_bytes, SMEM_MAX) - 1024 - 512 - self.NT * TB
        n = min(8, avail // TB)
        if n < 4:
            raise TemplateMismatch("meta smem_bytes too small for 2+2 K/V stages")
        self.SK, self.SV = (n + 1) // 2, n // 2
        self.split_p = bool(cls.SPLIT_P.get(D, False)) and self.NT * (128 + 64 + D) <= 512
        self.pair = (bool(cls.PAIR.get(D, False)) and not self.split_p and self.NT == 2
                     and (S // 256) % 2 == 0 and tuple(ctx.grid[1:]) == (1, 1))
        if self.pair:
            # K and V stages hold half a block each: twice as many fit
            n = min(12, avail // (TB // 2))
            self.SK, self.SV = (n + 1) // 2, n // 2
        return self

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        ctx = self.ctx
        D, S, NT = self.D, self.S, self.NT
        NB = S // 128                      # key blocks
        QB = S // (128 * NT)               # CTAs per (batch, head)
        TB = self.tile_bytes               # one 128 x D bf16 tile
        NBX = D // 64                      # 64-column boxes per tile
        pair = self.pair
        TBK = TB // 2 if pair else TB      # a K stage: 64 or 128 keys x D
        TBV = TB // 2 if pair else TB      # a V stage: 128 keys x D/2 or D columns
        KBOX = 64 * 128 if pair else 128 * 128   # bytes of one 64-column K box
        params = ctx.params() + [("tmapQ", ".align 64 .b8", "[128]"),
                                 ("tmapK", ".align 64 .b8", "[128]"),
                                 ("tmapV", ".align 64 .b8", "[128]")]
        k = Kernel(ctx.entry, params)
        k.maxntid = (512, 1, 1)
        if pair:
            k.reqnctapercluster = (2, 1, 1)
            k.directive("cluster 2 1 1")
        k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
        k.decl(".global .align 4 .u32 __emmy_status;")
        rows = self.B * self.H * S
        for nm, buf in (("tmapQ", self.q), ("tmapK", self.k), ("tmapV", self.v)):
            bk = 64 if pair and nm == "tmapK" else 128
            k.directive(f"tmap {nm} buf={buf} dtype=9 dims={D},{rows} strides={D * 2} "
                        f"box=64,{bk} swizzle=3")
        k.comment(f"emmy-b200 template: tcgen05 flash attention B={self.B} H={self.H} S={S} "
                  f"D={D}, {NT} query tile(s) per CTA")
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
        k(f"mad.lo.u32 {qrow0}, {qb}, {128 * NT}, {krow0};")
        SK, SV = self.SK, self.SV
        if pair:
            rank = k.special("%cluster_ctarank")
            plead = k.reg("p")
            k(f"setp.eq.u32 {plead}, {rank}, 0;")
        # shared memory: Q tiles | K ring (SK tiles) | V ring (SV tiles) |
        # barriers | tmem slot
        raw = k.reg("r")
        k(f"mov.u32 {raw}, __emmy_smem;")
        qs = k.reg("r")
        k(f"add.u32 {qs}, {raw}, 1023;")
        k(f"and.b32 {qs}, {qs}, -1024;")
        kring = k.reg("r")
        k(f"add.u32 {kring}, {qs}, {NT * TB};")
        vring = k.reg("r")
        k(f"add.u32 {vring}, {kring}, {SK * TBK};")
        bars = k.reg("r")
        k(f"add.u32 {bars}, {vring}, {SV * TBV};")
        # barrier slots
        Q_FULL = 0
        K_FULL, K_EMPTY = 1, 1 + SK
        V_FULL, V_EMPTY = 1 + 2 * SK, 1 + 2 * SK + SV
        S_FULL = V_EMPTY + SV          # [NT]: scores of tile t ready (tcgen05.commit)
        P_READY = S_FULL + NT          # [NT]: the 4 softmax warps wrote P of tile t
        FINAL = P_READY + NT           # [NT]: last P V of tile t done
        split = self.split_p
        # split P: the tiles share S_FULL, P_READY (4 NT arrivals) and S_FREE
        # (4 NT arrivals: every softmax warp has read its S), and one commit
        # per block on DONE[j % R] marks block j's P V (and, MMAs completing in
        # order, the Q K^T of block j+1 before it) complete: the K and V
        # producers, the softmax's reuse of P and O and the epilogue all wait
        # on that ring (R >= each ring's depth keeps their waits within one
        # phase of the barrier they read)
        S_FREE = FINAL + NT
        R = max(SK, SV)
        DONE = S_FREE + NT
        DRAIN = DONE + (R if split else 0)   # the MMA thread's own ops in flight at exit
        NSLOT = DRAIN + 1
        assert NSLOT * 8 + 4 <= 512
        tslot = k.reg("r")
        k(f"add.u32 {tslot}, {bars}, {NSLOT * 8};")
        status = k.reg("rd")
        k(f"mov.u64 {status}, __emmy_status;")
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip = k.label("SKIP_INIT")
        k(f"@!{p0} bra {skip};")
        for slot in range(NSLOT):
            if split:
                cnt = 4 * NT if slot in (P_READY, S_FREE) else 1
            else:
                # pair: the leader's P_READY counts both CTAs' softmax warps
                cnt = (8 if pair else 4) if P_READY <= slot < P_READY + NT else 1

            k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * slot}], {cnt};")
        k("fence.mbarrier_init.release.cluster;")
        for r in (tq, tk, tv):
            k(f"prefetch.tensormap [{r}];")
        k.mark(skip)
        pwm = k.reg("p")
        k(f"setp.eq.u32 {pwm}, {warp}, {MMA_WARP};")
        skip2 = k.label("SKIP_ALLOC")
        k(f"@!{pwm} bra {skip2};")
        cg = "cta_group::2" if pair else "cta_group::1"
        # a pair allocates collectively: the same 512 columns in both CTAs
        k(f"tcgen05.alloc.{cg}.sync.aligned.shared::cta.b32 [{tslot}], 512;")
        k(f"tcgen05.relinquish_alloc_permit.{cg}.sync.aligned;")
        k.mark(skip2)
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
        if pair:
            # both CTAs' barriers and tensor memory exist before any cross-CTA use
            k("barrier.cluster.arrive.release.aligned;")
            k("barrier.cluster.wait.acquire.aligned;")
        k("tcgen05.fence::after_thread_sync;")
        tmem = k.reg("r")
        k(f"ld.shared.u32 {tmem}, [{tslot}];")
        # register split: the softmax warpgroups (one row of scores each in
        # registers) take SOFT_REGS, the others give theirs up; the launch
        # holds exactly 512 x LAUNCH_REGS (.maxnreg with setmaxnreg makes
        # ptxas allocate exactly that), and the shares add up to no more
        shares = [SOFT_REGS if g_ < NT else ROLE_REGS for g_ in range(4)]
        assert sum(128 * r for r in shares) <= 512 * LAUNCH_REGS
        k.maxnreg = LAUNCH_REGS
        k.directive(f"regsplit launch={LAUNCH_REGS} threads=512 "
                    f"warpgroups={','.join(str(r) for r in shares)}")
        pl0 = k.reg("p")
        k(f"setp.eq.u32 {pl0}, {lane}, 0;")
        # the softmax warps branch to their code, which setmaxnreg.inc
        # dominates; everyone else gives up registers first.  The two regions
        # never merge again (each ends in its own barrier and exit): code
        # reached from both would need one register assignment valid under
        # both limits
        pwg = k.reg("p")
        k(f"setp.lt.u32 {pwg}, {warp}, {4 * NT};")
        soft_entry = k.label("SOFTMAX")
        k(f"@{pwg} bra {soft_entry};")
        k(f"setmaxnreg.dec.sync.aligned.u32 {ROLE_REGS};")
        teardown = k.label("TEARDOWN")
        soft_teardown = k.label("SOFT_TEARDOWN")
        wait = GemmTemplate._wait

        def bar(slot, idx=None):
            """Address of barrier ``slot`` (+ a register index)."""
            r = k.reg("r")
            if idx is None:
                k(f"add.u32 {r}, {bars}, {8 * slot};")
            else:
                k(f"mad.lo.u32 {r}, {idx}, 8, {bars};")
                k(f"add.u32 {r}, {r}, {8 * slot};")
            return r

        def ring_slot(jreg, depth):
            """(stage, phase) of block j in a ring of ``depth`` stages."""
            st_ = k.reg("r")
            k(f"rem.u32 {st_}, {jreg}, {depth};")
            ph_ = k.reg("r")
            k(f"div.u32 {ph_}, {jreg}, {depth};")
            k(f"and.b32 {ph_}, {ph_}, 1;")
            return st_, ph_

        if pair:
            cmask = k.reg("h")
            k(f"mov.b16 {cmask}, 3;")

        def commit(addr, local=False):
            """Arrive on ``addr`` once this thread's MMAs so far complete; a
            pair's leader signals the barrier at that offset in both CTAs."""
            if pair and not local:
                k(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster"
                  f".multicast::cluster.b64 [{addr}], {cmask};")
            elif pair:
                k(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [{addr}];")
            else:
                k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
                  f"[{addr}];")

        j = k.reg("r")

        def producer(which, warp_id, tmap, ring, depth, full, empty, load_q):
            pp = k.reg("p")
            k(f"setp.eq.u32 {pp}, {warp}, {warp_id};")
            k(f"and.pred {pp}, {pp}, {pl0};")
            end_p = k.label(f"END_{which}")
            k(f"@!{pp} bra {end_p};")
            # a pair's copies complete on the LEADER's barriers (mapa address),
            # which the leader arms with both CTAs' bytes
            cpy = ("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier"
                   "::complete_tx::bytes" if pair else
                   "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes")
            arm = f"@{plead} " if pair else ""
            ncta = 2 if pair else 1

            def target(addr):
                if not pair:
                    return addr
                r = k.reg("r")
                k(f"mapa.shared::cluster.u32 {r}, {addr}, 0;")
                return r
            if load_q:
                qf = bar(Q_FULL)
                k(f"{arm}mbarrier.arrive.expect_tx.shared::cta.b64 _, [{qf}], {ncta * NT * TB};")
                qft = target(qf)
                for t in range(NT):
                    qr = k.reg("r")
                    k(f"add.u32 {qr}, {qrow0}, {128 * t};")
                    for i in range(NBX):
                        k(f"{cpy} [{qs}+{t * TB + i * 16384}], [{tq}, {{{64 * i}, {qr}}}], "
                          f"[{qft}];")
            k(f"mov.u32 {j}, 0;")
            top = k.label(f"PROD_{which}")
            k.mark(top)
            st_, ph_ = ring_slot(j, depth)
            if split:
                # the stage's previous block b = j - depth is free once the
                # P V iteration that last read it is done: V(b) -> DONE(b);
                # K(b) (read by the Q K^T of iteration b-1) -> DONE(max(b-1, 0))
                nowait = k.label(f"NOWAIT_{which}")
                pf = k.reg("p")
                k(f"setp.lt.u32 {pf}, {j}, {depth};")
                k(f"@{pf} bra {nowait};")
                n_ = k.reg("r")
                k(f"sub.u32 {n_}, {j}, {depth + (1 if which == 'K' else 0)};")
                k(f"max.s32 {n_}, {n_}, 0;")
                ds, dph = ring_slot(n_, R)
                wait(k, bar(DONE, ds), dph, status, 1, end_p)
                k.mark(nowait)
            else:
                par = k.reg("r")
                k(f"xor.b32 {par}, {ph_}, 1;")
                wait(k, bar(empty, st_), par, status, 1, end_p)
            kr = k.reg("r")
            k(f"mad.lo.u32 {kr}, {j}, 128, {krow0};")
            stage = TBK if which == "K" else TBV
            dst = k.reg("r")
            k(f"mad.lo.u32 {dst}, {st_}, {stage}, {ring};")
            fb = bar(full, st_)
            k(f"{arm}mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {ncta * stage};")
            fbt = target(fb)
            if pair and which == "K":
                # this CTA's 64 keys of the block, all D columns
                k(f"mad.lo.u32 {kr}, {rank}, 64, {kr};")
                for i in range(NBX):
                    k(f"{cpy} [{dst}+{i * KBOX}], [{tmap}, {{{64 * i}, {kr}}}], [{fbt}];")
            elif pair:
                # all 128 keys of the block, this CTA's D/2 columns
                c0 = k.reg("r")
                k(f"mul.lo.u32 {c0}, {rank}, {D // 2};")
                for i in range(NBX // 2):
                    ci = k.reg("r")
                    k(f"add.u32 {ci}, {c0}, {64 * i};")
                    k(f"{cpy} [{dst}+{i * 16384}], [{tmap}, {{{ci}, {kr}}}], [{fbt}];")
            else:
                for i in range(NBX):
                    k(f"{cpy} [{dst}+{i * 16384}], [{tmap}, {{{64 * i}, {kr}}}], [{fbt}];")
            k.comment(f"@trace {10 if load_q else 11} {j}")
            k(f"add.u32 {j}, {j}, 1;")
            pl = k.reg("p")
            k(f"setp.lt.u32 {pl}, {j}, {NB};")
            k(f"@{pl} bra {top};")
            k.mark(end_p)

        # ---------------- producers: Q and K on one warp, V on another ----------------
        producer("K", PROD_K_WARP, tk, kring, SK, K_FULL, K_EMPTY, True)
        producer("V", PROD_V_WARP, tv, vring, SV, V_FULL, V_EMPTY, False)

        # ---------------- MMA issuer ----------------
        pm = k.reg("p")
        k(f"setp.eq.u32 {pm}, {warp}, {MMA_WARP};")
        k(f"and.pred {pm}, {pm}, {pl0};")
        if pair:
            k(f"and.pred {pm}, {pm}, {plead};")      # the leader's thread issues for both
        end_mma = k.label("END_MMA")
        skip_mma = k.label("SKIP_MMA")
        k(f"@!{pm} bra {skip_mma};")
        MM = 256 if pair else 128                    # rows per MMA: a pair's both tiles
        iqk = k.reg("r")
        k(f"mov.u32 {iqk}, {idesc_mma(MM, 128, False)};")
        ipv = k.reg("r")
        k(f"mov.u32 {ipv}, {idesc_mma(MM, D, True)};")
        hiK = _desc_hi(16, 1024)
        hiV = _desc_hi(16384, 1024)
        ptrue = k.reg("p")
        k(f"setp.eq.u32 {ptrue}, 0, 0;")
        pfalse = k.reg("p")
        k(f"setp.ne.u32 {pfalse}, 0, 0;")
        zero = k.reg("r")
        k(f"mov.u32 {zero}, 0;")
        wait(k, bar(Q_FULL), zero, status, 2, end_mma)
        dq = []
        for t in range(NT):
            qa = k.reg("r")
            k(f"add.u32 {qa}, {qs}, {t * TB};")
            dq.append(GemmTemplate._desc(k, qa, hiK))

        def k_ready(jreg):
            """Wait for K block ``jreg``; return (its descriptor, its stage)."""
            kst, kph = ring_slot(jreg, SK)
            wait(k, bar(K_FULL, kst), kph, status, 2, end_mma)
            k("tcgen05.fence::after_thread_sync;")
            kad = k.reg("r")
            k(f"mad.lo.u32 {kad}, {kst}, {TBK}, {kring};")
            return GemmTemplate._desc(k, kad, hiK), kst

        def issue_qk(t, dk, jreg, do_commit=True):
            """S_t = Q_t K^T (overwrites the tile's score buffer)."""
            for kk in range(D // 16):
                off = (kk % 4) * 2 + (kk // 4) * 1024        # +32 B along K; next box
                offk = (kk % 4) * 2 + (kk // 4) * (KBOX // 16)
                a = k.reg("rd")
                k(f"add.s64 {a}, {dq[t]}, {off};")
                bd = k.reg("rd")
                k(f"add.s64 {bd}, {dk}, {offk};")
                k(f"tcgen05.mma.{cg}.kind::f16 [{s_tm[t]}], {a}, {bd}, {iqk}, "
                  f"{pfalse if kk == 0 else ptrue};")
            if do_commit:
                commit(bar(S_FULL + t))
            k.comment(f"@trace {3 * t} {jreg}")

        def issue_pv(t, dv, pacc):
            """O_t += P_t V (P: the tile's own 64 columns with split P, else the
            first 64 columns of the score buffer)."""
            for kk in range(8):                     # 128 keys, K=16 per MMA
                a = k.reg("r")
                k(f"add.u32 {a}, {p_tm[t]}, {8 * kk};")  # 16 bf16 = 8 TMEM columns
                bd = k.reg("rd")
                k(f"add.s64 {bd}, {dv}, {kk * 128};")   # +16 key rows * 128 B
                k(f"tcgen05.mma.{cg}.kind::f16 [{o_tm[t]}], [{a}], {bd}, {ipv}, "
                  f"{pacc if kk == 0 else ptrue};")

        s_tm, o_tm, p_tm = [], [], []
        for t in range(NT):
            r1 = k.reg("r")
            k(f"add.u32 {r1}, {tmem}, {128 * t};")
            s_tm.append(r1)
            r2 = k.reg("r")
            k(f"add.u32 {r2}, {tmem}, {(128 + 64) * NT + D * t if split else 256 + D * t};")
            o_tm.append(r2)
            if split:
                r3 = k.reg("r")
                k(f"add.u32 {r3}, {tmem}, {128 * NT + 64 * t};")
                p_tm.append(r3)
            else:
                p_tm.append(r1)
        # block 0 scores of every tile
        k(f"mov.u32 {j}, 0;")
        dk0, kst0 = k_ready(j)
        for t in range(NT):
            issue_qk(t, dk0, j, not split)
        if split:
            commit(bar(S_FULL))
        else:
            commit(bar(K_EMPTY, kst0))
        jn = k.reg("r")
        pacc = k.reg("p")
        par = k.reg("r")

        def block(last: bool):
            """P V of block j for every tile, each followed (unless ``last``)
            by that tile's scores of block j+1."""
            vst, vph = ring_slot(j, SV)
            wait(k, bar(V_FULL, vst), vph, status, 2, end_mma)
            k.comment(f"@trace 8 {j}")
            k("tcgen05.fence::after_thread_sync;")
            vad = k.reg("r")
            k(f"mad.lo.u32 {vad}, {vst}, {TBV}, {vring};")
            dv = GemmTemplate._desc(k, vad, hiV)
            k(f"setp.ne.u32 {pacc}, {j}, 0;")
            k(f"and.b32 {par}, {j}, 1;")
            dk = kst = None
            if not last and self.EARLY_K:
                # the next K block (loaded stages ahead) before the P waits:
                # its wait and descriptor stay off the tiles' critical path
                k(f"add.u32 {jn}, {j}, 1;")
                dk, kst = k_ready(jn)
                k.comment(f"@trace 9 {jn}")
            for t in range(NT):
                wait(k, bar(P_READY + t), par, status, 2, end_mma,
                     ".acquire.cluster" if pair else "")
                k.comment(f"@trace {3 * t + 1} {j}")
                k("tcgen05.fence::after_thread_sync;")
                issue_pv(t, dv, pacc)
                k.comment(f"@trace {3 * t + 2} {j}")
                if last:
                    commit(bar(FINAL + t))
                else:
                    if t == 0 and dk is None:
                        k(f"add.u32 {jn}, {j}, 1;")
                        dk, kst = k_ready(jn)
                        k.comment(f"@trace 9 {jn}")
                    issue_qk(t, dk, jn)
            commit(bar(V_EMPTY, vst))
            if not last:
                commit(bar(K_EMPTY, kst))

        def block_split(last: bool):
            """Split P: once every softmax warp has read S of block j, the
            scores of block j+1 for both tiles (one commit on the shared
            S_FULL); once every softmax warp has stored P of block j, P V of
            block j for both tiles and one commit on DONE[j % R]."""
            k(f"and.b32 {par}, {j}, 1;")
            if not last:
                k(f"add.u32 {jn}, {j}, 1;")
                dk, kst = k_ready(jn)
                k.comment(f"@trace 9 {jn}")
                wait(k, bar(S_FREE), par, status, 2, end_mma)
                k("tcgen05.fence::after_thread_sync;")
                for t in range(NT):
                    issue_qk(t, dk, jn, False)
                k.comment(f"@trace 0 {jn}")
                commit(bar(S_FULL))
            vst, vph = ring_slot(j, SV)
            wait(k, bar(V_FULL, vst), vph, status, 2, end_mma)
            k.comment(f"@trace 8 {j}")
            vad = k.reg("r")
            k(f"mad.lo.u32 {vad}, {vst}, {TBV}, {vring};")
            dv = GemmTemplate._desc(k, vad, hiV)
            k(f"setp.ne.u32 {pacc}, {j}, 0;")
            wait(k, bar(P_READY), par, status, 2, end_mma)
            k.comment(f"@trace 1 {j}")
            k("tcgen05.fence::after_thread_sync;")
            for t in range(NT):
                issue_pv(t, dv, pacc)
            k.comment(f"@trace 2 {j}")
            ds_ = k.reg("r")
            k(f"rem.u32 {ds_}, {j}, {R};")
            commit(bar(DONE, ds_))

        if split:
            block = block_split  # noqa: F811
        if NB > 1:
            top2 = k.label("MMA")
            k.mark(top2)
            block(False)
            k(f"add.u32 {j}, {j}, 1;")
            pl2 = k.reg("p")
            k(f"setp.lt.u32 {pl2}, {j}, {NB - 1};")
            k(f"@{pl2} bra {top2};")
        k(f"mov.u32 {j}, {NB - 1};")
        block(True)
        k.mark(end_mma)
        # wait (bounded) for this thread's tensor-core operations still in
        # flight, so that no MMA outlives the TMEM allocation on an error path
        commit(bar(DRAIN), local=True)
        wait(k, bar(DRAIN), zero, status, 6, skip_mma)
        k.mark(skip_mma)
        k(f"bra {teardown};")

        # ------------- softmax warps 0..4*NT-1: one thread per query row -------------
        k.mark(soft_entry)
        k(f"setmaxnreg.inc.sync.aligned.u32 {SOFT_REGS};")
        end_sm = k.label("END_SM")
        q4 = k.reg("r")
        k(f"and.b32 {q4}, {warp}, 3;")
        tt = k.reg("r")                            # query tile of this warp
        k(f"shr.u32 {tt}, {warp}, 2;")
        row = k.reg("r")
        k(f"mad.lo.u32 {row}, {q4}, 32, {lane};")
        trow = k.reg("r")
        k(f"shl.b32 {trow}, {q4}, 21;")            # TMEM lane field (32*q4) << 16
        k(f"add.u32 {trow}, {trow}, {tmem};")
        srow = k.reg("r")
        k(f"mad.lo.u32 {srow}, {tt}, 128, {trow};")
        orow_tm = k.reg("r")
        k(f"mad.lo.u32 {orow_tm}, {tt}, {D}, {trow};")
        k(f"add.u32 {orow_tm}, {orow_tm}, {(128 + 64) * NT if split else 256};")
        prow = srow
        if split:
            prow = k.reg("r")
            k(f"mad.lo.u32 {prow}, {tt}, 64, {trow};")
            k(f"add.u32 {prow}, {prow}, {128 * NT};")
        sfull = k.reg("r")
        k(f"mad.lo.u32 {sfull}, {tt}, 8, {bars};")
        pready = k.reg("r")
        k(f"add.u32 {pready}, {sfull}, {8 * P_READY};")
        fin = k.reg("r")
        k(f"add.u32 {fin}, {sfull}, {8 * FINAL};")
        sfree = k.reg("r")
        k(f"add.u32 {sfree}, {sfull}, {8 * S_FREE};")
        k(f"add.u32 {sfull}, {sfull}, {8 * S_FULL};")
        if split:     # barriers shared by the tiles; fin = the DONE ring
            k(f"add.u32 {pready}, {bars}, {8 * P_READY};")
            k(f"add.u32 {sfree}, {bars}, {8 * S_FREE};")
            k(f"add.u32 {sfull}, {bars}, {8 * S_FULL};")
            k(f"add.u32 {fin}, {bars}, {8 * DONE};")
        sc = k.reg("f")
        k(f"ld.global.nc.f32 {sc}, [{sbuf}];")
        k(f"rcp.rn.f32 {sc}, {sc};")
        k(f"mul.rn.f32 {sc}, {sc}, 0f{_f32hex(LOG2E)};")     # c = s * log2(e)
        sc2 = k.reg("rd")
        k(f"mov.b64 {sc2}, {{{sc}, {sc}}};")
        cst = {}
        for nm, val in (("magic", 0x4B400000), ("clamp", _bits(-126.0))) + tuple(
                (f"c{i}", _bits(c)) for i, c in enumerate(EXP2_POLY)):
            r = k.reg("rd" if nm != "clamp" else "f")
            k(f"mov.b64 {r}, 0x{val:08X}{val:08X};" if nm != "clamp" else f"mov.b32 {r}, 0x{val:08X};")
            cst[nm] = r
        poly = self.poly_pairs()
        m = k.reg("f")                             # max used for the exponents
        k(f"mov.f32 {m}, 0fFF800000;")
        lsum = k.reg("f")
        k(f"mov.f32 {lsum}, 0f00000000;")
        k(f"mov.u32 {j}, 0;")
        top3 = k.label("SMX")
        k.mark(top3)
        spar = k.reg("r")
        k(f"and.b32 {spar}, {j}, 1;")
        wait(k, sfull, spar, status, 3, soft_teardown)
        k.comment(f"@trace 6 {j}")
        k("tcgen05.fence::after_thread_sync;")

        def ld32(col):
            regs = k.regs("r", 32)
            k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{srow}+{col}];")
            return regs

        def wait_ld():
            k("tcgen05.wait::ld.sync.aligned;")

        def max_into(mx, vals, first):
            """Fold ``vals`` into the eight partial maxima (3-input max)."""
            rest = list(vals)
            if first:
                for i in range(8):
                    k(f"max.f32 {mx[i]}, {rest[i]}, {rest[i + 8]}, {rest[i + 16]};")
                rest = rest[24:]
            for i in range(0, len(rest), 2):
                k(f"max.f32 {mx[(i // 2) % 8]}, {mx[(i // 2) % 8]}, {rest[i]}, {rest[i + 1]};")

        def exp_pack(vals, negm2, ps2):
            """p = 2^(s*c - m) of 32 scores (f32 pairs), summed into ``ps2``;
            returns 16 bf16 pairs.  Pairs in ``poly`` evaluate 2^x on the FMA
            pipe instead of the MUFU."""
            packed = k.regs("r", 16)
            for pi in range(16):
                x2 = k.reg("rd")
                k(f"mov.b64 {x2}, {{{vals[2 * pi]}, {vals[2 * pi + 1]}}};")
                k(f"fma.rn.f32x2 {x2}, {x2}, {sc2}, {negm2};")
                e0, e1 = k.reg("f"), k.reg("f")
                if pi in poly:
                    self._exp2_poly(k, x2, e0, e1, cst)
                else:
                    t0, t1 = k.reg("f"), k.reg("f")
                    k(f"mov.b64 {{{t0}, {t1}}}, {x2};")
                    k(f"ex2.approx.ftz.f32 {e0}, {t0};")
                    k(f"ex2.approx.ftz.f32 {e1}, {t1};")
                e2 = k.reg("rd")
                k(f"mov.b64 {e2}, {{{e0}, {e1}}};")
                k(f"add.rn.f32x2 {ps2[pi % 4]}, {ps2[pi % 4]}, {e2};")
                k(f"cvt.rn.bf16x2.f32 {packed[pi]}, {e1}, {e0};")
            return packed

        def st16(col, pk):
            k(f"tcgen05.st.sync.aligned.32x32b.x16.b32 [{prow}+{col}], {{{', '.join(pk)}}};")

        def rescale_o(factor):
            """O row *= factor in TMEM (32 columns at a time)."""
            f2 = k.reg("rd")
            k(f"mov.b64 {f2}, {{{factor}, {factor}}};")
            for c in range(D // 32):
                ov = k.regs("r", 32)
                k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, "
                  f"[{orow_tm}+{32 * c}];")
                wait_ld()
                self._scale_pairs(k, ov, f2)
                k(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{orow_tm}+{32 * c}], "
                  f"{{{', '.join(ov)}}};")

        if pair:
            # the P_READY the leader's issuing thread waits on
            lpready = k.reg("r")
            k(f"mapa.shared::cluster.u32 {lpready}, {pready}, 0;")

        def p_ready_arrive():
            """This warp's P (and O) stores are complete: one arrival per warp
            on the tile's P_READY barrier (lane 0, after the warp converges);
            in a pair, on the leader's, with release semantics for the
            cluster (the leader's MMA reads this CTA's TMEM)."""
            k("tcgen05.wait::st.sync.aligned;")
            k("tcgen05.fence::before_thread_sync;")
            k("bar.warp.sync 0xffffffff;")
            if pair:
                k(f"@{pl0} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{lpready}];")
            else:
                k(f"@{pl0} mbarrier.arrive.shared::cta.b64 _, [{pready}];")

        def row_sum(ps2):
            k(f"add.rn.f32x2 {ps2[0]}, {ps2[0]}, {ps2[1]};")
            k(f"add.rn.f32x2 {ps2[2]}, {ps2[2]}, {ps2[3]};")
            k(f"add.rn.f32x2 {ps2[0]}, {ps2[0]}, {ps2[2]};")
            s0, s1 = k.reg("f"), k.reg("f")
            k(f"mov.b64 {{{s0}, {s1}}}, {ps2[0]};")
            k(f"add.rn.f32 {s0}, {s0}, {s1};")
            return s0

        if split:
            self._softmax_split(k, dict(
                ld32=ld32, wait_ld=wait_ld, st16=st16, rescale_o=rescale_o,
                p_ready_arrive=p_ready_arrive, row_sum=row_sum, max_into=max_into, sc=sc,
                sc2=sc2, cst=cst, poly=poly, m=m, lsum=lsum, j=j, top3=top3, sfree=sfree,
                fin=fin, pl0=pl0, NB=NB, R=R, status=status, fail=soft_teardown, wait=wait))
        else:
            # the row's 128 scores stay in registers for the whole block
            sv = ld32(0) + ld32(32) + ld32(64) + ld32(96)
            wait_ld()
            k.comment(f"@trace 12 {j}")
            ps2 = [k.reg("rd") for _ in range(4)]      # row-sum partials, f32 pairs
            negm = k.reg("f")
            negm2 = k.reg("rd")
            mx = [k.reg("f") for _ in range(8)]

            def p_pass(base, fold_max):
                """P = 2^(s*c - base) of the 128 scores over S columns 0..63 (P of
                32-column chunk c at 16c), summed into ``ps2``; with ``fold_max``
                the row max is folded into ``mx`` on the way (it does not feed the
                exponentials).  One software-pipelined stream over the 64 column
                pairs: step s issues the scale of pair s+1, the exponentials of
                pair s, the sum and bf16 pack of pair s-2 and one max, so the FMA
                and ALU work issues while the MUFU works through the ex2s."""
                k(f"neg.f32 {negm}, {base};")
                k(f"mov.b64 {negm2}, {{{negm}, {negm}}};")
                for r in ps2:
                    k(f"mov.b64 {r}, 0;")
                LEAD, LAG = self.PIPE
                t2, es = {}, {}
                packed = {}
                maxops = []
                if fold_max:
                    for i in range(8):
                        maxops.append((mx[i], sv[i], sv[i + 8], sv[i + 16]))
                    rest = sv[24:]
                    for i in range(0, len(rest), 2):
                        slot = mx[(i // 2) % 8]
                        maxops.append((slot, slot, rest[i], rest[i + 1]))

                def stage_a(q):
                    x2 = k.reg("rd")
                    k(f"mov.b64 {x2}, {{{sv[2 * q]}, {sv[2 * q + 1]}}};")
                    k(f"fma.rn.f32x2 {x2}, {x2}, {sc2}, {negm2};")
                    t2[q] = x2

                def stage_b(q):
                    e0, e1 = k.reg("f"), k.reg("f")
                    if q % 16 in poly:
                        self._exp2_poly(k, t2.pop(q), e0, e1, cst)
                    else:
                        a0, a1 = k.reg("f"), k.reg("f")
                        k(f"mov.b64 {{{a0}, {a1}}}, {t2.pop(q)};")
                        k(f"ex2.approx.ftz.f32 {e0}, {a0};")
                        k(f"ex2.approx.ftz.f32 {e1}, {a1};")
                    es[q] = (e0, e1)

                def stage_c(q):
                    e0, e1 = es.pop(q)
                    e2 = k.reg("rd")
                    k(f"mov.b64 {e2}, {{{e0}, {e1}}};")
                    k(f"add.rn.f32x2 {ps2[q % 4]}, {ps2[q % 4]}, {e2};")
                    c, pi = divmod(q, 16)
                    if pi == 0:
                        packed[c] = k.regs("r", 16)
                    k(f"cvt.rn.bf16x2.f32 {packed[c][pi]}, {e1}, {e0};")
                    if pi == 15:
                        st16(16 * c, packed.pop(c))

                for q in range(LEAD):
                    stage_a(q)
                for st_ in range(64 + LAG):
                    if st_ + LEAD < 64:
                        stage_a(st_ + LEAD)
                    if st_ < 64:
                        stage_b(st_)
                    if st_ - LAG >= 0:
                        stage_c(st_ - LAG)
                    if maxops:
                        d_, a_, b_, c_ = maxops.pop(0)
                        k(f"max.f32 {d_}, {a_}, {b_}, {c_};")
                assert not maxops and not t2 and not es and not packed

            # speculative pass against the current base m; it stands unless a row
            # max grew by more than 2^8 (lazy rescaling: p stays <= 256, and the
            # final 1/l uses the same base, so this is exact)
            p_pass(m, True)
            k(f"max.f32 {mx[0]}, {mx[0]}, {mx[1]}, {mx[2]};")
            k(f"max.f32 {mx[3]}, {mx[3]}, {mx[4]}, {mx[5]};")
            k(f"max.f32 {mx[6]}, {mx[6]}, {mx[7]}, {mx[0]};")
            k(f"max.f32 {mx[0]}, {mx[3]}, {mx[6]};")
            cand = k.reg("f")
            k(f"mul.rn.f32 {cand}, {mx[0]}, {sc};")
            thr = k.reg("f")
            k(f"add.rn.f32 {thr}, {m}, 0f41000000;")         # m + 8
            need = k.reg("p")
            k(f"setp.gt.f32 {need}, {cand}, {thr};")
            anyw = k.reg("p")
            k(f"vote.sync.any.pred {anyw}, {need}, 0xffffffff;")
            fast = k.label("P_FAST")
            k(f"@!{anyw} bra {fast};")
            # slow path (always on the first block): new base, P again from the
            # scores in registers, l and this warp's running O rows rescaled by
            # 2^(m_old - m_new) (the tile's previous P V completed before its
            # scores were released; the first block's O is not yet written)
            meff = k.reg("f")
            k(f"selp.f32 {meff}, {cand}, {m}, {need};")
            alpha = k.reg("f")
            dlt = k.reg("f")
            k(f"sub.rn.f32 {dlt}, {m}, {meff};")
            k(f"ex2.approx.ftz.f32 {alpha}, {dlt};")
            k(f"@!{need} mov.f32 {alpha}, 0f3F800000;")
            p_pass(meff, False)
            skip_rs = k.label("NO_RESCALE")
            pj0 = k.reg("p")
            k(f"setp.eq.u32 {pj0}, {j}, 0;")
            k(f"@{pj0} bra {skip_rs};")
            rescale_o(alpha)
            k.mark(skip_rs)
            k(f"mul.rn.f32 {lsum}, {lsum}, {alpha};")
            k(f"mov.f32 {m}, {meff};")
            k.mark(fast)
            p_ready_arrive()
            k.comment(f"@trace 7 {j}")
            rsum = row_sum(ps2)
            k(f"add.rn.f32 {lsum}, {lsum}, {rsum};")
            k(f"add.u32 {j}, {j}, 1;")
            pl3 = k.reg("p")
            k(f"setp.lt.u32 {pl3}, {j}, {NB};")
            k(f"@{pl3} bra {top3};")
        # epilogue: O row * (1 / l) -> global
        if split:
            # the last block's P V: DONE[(NB-1) % R], its ((NB-1) // R)-th completion
            fl = k.reg("r")
            k(f"add.u32 {fl}, {fin}, {8 * ((NB - 1) % R)};")
            wait(k, fl, ((NB - 1) // R) & 1, status, 3, soft_teardown)
        else:
            wait(k, fin, self._zero(k), status, 3, soft_teardown)
        k("tcgen05.fence::after_thread_sync;")
        inv = k.reg("f")
        k(f"rcp.rn.f32 {inv}, {lsum};")
        inv2 = k.reg("rd")
        k(f"mov.b64 {inv2}, {{{inv}, {inv}}};")
        grow = k.reg("r")
        k(f"mad.lo.u32 {grow}, {tt}, 128, {row};")
        k(f"add.u32 {grow}, {grow}, {qrow0};")
        oa = k.reg("rd")
        k(f"mul.wide.u32 {oa}, {grow}, {D * 4};")
        k(f"add.s64 {oa}, {oa}, {obase};")
        for c in range(D // 32):
            regs = k.regs("r", 32)
            k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, "
              f"[{orow_tm}+{32 * c}];")
            wait_ld()
            self._scale_pairs(k, regs, inv2)
            for v8 in range(4):
                k(f"st.global.v8.b32 [{oa}+{128 * c + 32 * v8}], "
                  f"{{{', '.join(regs[8 * v8:8 * v8 + 8])}}};")
        k.mark(end_sm)
        k.mark(soft_teardown)
        k("tcgen05.fence::before_thread_sync;")
        k("barrier.sync 0;")
        if pair:   # the peer may still use this CTA's memory until it arrives too
            k("barrier.cluster.arrive.release;")
            k("barrier.cluster.wait.acquire;")
        k("ret;")

        # ---------------- teardown of the other warps ----------------
        k.mark(teardown)
        k("tcgen05.fence::before_thread_sync;")
        k("barrier.sync 0;")
        if pair:
            k("barrier.cluster.arrive.release;")
            k("barrier.cluster.wait.acquire;")
        end = k.label("END")
        k(f"@!{pwm} bra {end};")
        k("bar.warp.sync 0xffffffff;")
        k("tcgen05.fence::after_thread_sync;")
        k(f"tcgen05.dealloc.{cg}.sync.aligned.b32 {tmem}, 512;")
        k.mark(end)
        k("ret;")
        return k.render()

    def _softmax_split(self, k, e):
        """The softmax warps' block body with split P (one thread per query
        row; S of block j already waited for):

        * the row's 128 scores are read from TMEM into registers and S is
          released at once (one arrival per warp on the tile's S_FREE), so the
          next block's Q K^T runs while this block's softmax works;
        * the row max, then the exponent base: it moves to the new max only
          when that exceeds it by more than 2^8 (lazy rescaling; always on the
          first block), with ``alpha = 2^(m_old - m_new)`` (exactly 1 for rows
          that keep their base);
        * ``p = 2^(s*c - m)`` of all 128 scores into 64 packed bf16 pairs held
          in registers, summed on the way;
        * the tile's previous P V must be complete before its P columns and O
          rows are touched (the tile's P_FREE barrier, one completion per
          block); then the O rows are rescaled by alpha if any row of the warp
          moved its base (never on the first block, before any P V), P is
          stored and the warp arrives on P_READY;
        * l = l * alpha + the row sum."""
        j, m, lsum = e["j"], e["m"], e["lsum"]
        sv = e["ld32"](0) + e["ld32"](32) + e["ld32"](64) + e["ld32"](96)
        e["wait_ld"]()
        k("tcgen05.fence::before_thread_sync;")
        k("bar.warp.sync 0xffffffff;")
        k(f"@{e['pl0']} mbarrier.arrive.shared::cta.b64 _, [{e['sfree']}];")
        k.comment(f"@trace 12 {j}")
        # row max: eight partial maxima (3-input max), then folded
        mx = [k.reg("f") for _ in range(8)]
        e["max_into"](mx, sv, True)
        k(f"max.f32 {mx[0]}, {mx[0]}, {mx[1]}, {mx[2]};")
        k(f"max.f32 {mx[3]}, {mx[3]}, {mx[4]}, {mx[5]};")
        k(f"max.f32 {mx[6]}, {mx[6]}, {mx[7]}, {mx[0]};")
        k(f"max.f32 {mx[0]}, {mx[3]}, {mx[6]};")
        k.comment(f"@trace 13 {j}")
        cand = k.reg("f")
        k(f"mul.rn.f32 {cand}, {mx[0]}, {e['sc']};")
        thr = k.reg("f")
        k(f"add.rn.f32 {thr}, {m}, 0f41000000;")         # m + 8
        need = k.reg("p")
        k(f"setp.gt.f32 {need}, {cand}, {thr};")
        anyw = k.reg("p")
        k(f"vote.sync.any.pred {anyw}, {need}, 0xffffffff;")
        meff = k.reg("f")
        k(f"selp.f32 {meff}, {cand}, {m}, {need};")
        alpha = k.reg("f")
        dlt = k.reg("f")
        k(f"sub.rn.f32 {dlt}, {m}, {meff};")           # 0 for rows that keep m
        k(f"ex2.approx.ftz.f32 {alpha}, {dlt};")
        k(f"mov.f32 {m}, {meff};")
        negm = k.reg("f")
        k(f"neg.f32 {negm}, {m};")
        negm2 = k.reg("rd")
        k(f"mov.b64 {negm2}, {{{negm}, {negm}}};")
        ps2 = [k.reg("rd") for _ in range(4)]      # row-sum partials, f32 pairs
        for r in ps2:
            k(f"mov.b64 {r}, 0;")
        LEAD, LAG = self.PIPE
        poly, cst, sc2 = e["poly"], e["cst"], e["sc2"]
        t2, es, packed = {}, {}, []

        def stage_a(q):
            x2 = k.reg("rd")
            k(f"mov.b64 {x2}, {{{sv[2 * q]}, {sv[2 * q + 1]}}};")
            k(f"fma.rn.f32x2 {x2}, {x2}, {sc2}, {negm2};")
            t2[q] = x2

        def stage_b(q):
            e0, e1 = k.reg("f"), k.reg("f")
            if q % 16 in poly:
                self._exp2_poly(k, t2.pop(q), e0, e1, cst)
            else:
                a0, a1 = k.reg("f"), k.reg("f")
                k(f"mov.b64 {{{a0}, {a1}}}, {t2.pop(q)};")
                k(f"ex2.approx.ftz.f32 {e0}, {a0};")
                k(f"ex2.approx.ftz.f32 {e1}, {a1};")
            es[q] = (e0, e1)

        def stage_c(q):
            e0, e1 = es.pop(q)
            e2 = k.reg("rd")
            k(f"mov.b64 {e2}, {{{e0}, {e1}}};")
            k(f"add.rn.f32x2 {ps2[q % 4]}, {ps2[q % 4]}, {e2};")
            pk = k.reg("r")
            k(f"cvt.rn.bf16x2.f32 {pk}, {e1}, {e0};")
            packed.append(pk)

        for q in range(LEAD):
            stage_a(q)
        for st_ in range(64 + LAG):
            if st_ + LEAD < 64:
                stage_a(st_ + LEAD)
            if st_ < 64:
                stage_b(st_)
            if st_ - LAG >= 0:
                stage_c(st_ - LAG)
        assert not t2 and not es and len(packed) == 64
        k.comment(f"@trace 14 {j}")
        # the tile's previous P V is done: its P columns and O rows are free
        skip_w = k.label("FIRST_BLOCK")
        pj0 = k.reg("p")
        k(f"setp.eq.u32 {pj0}, {j}, 0;")
        k(f"@{pj0} bra {skip_w};")
        jp = k.reg("r")
        k(f"sub.u32 {jp}, {j}, 1;")                  # DONE of block j-1
        ds = k.reg("r")
        k(f"rem.u32 {ds}, {jp}, {e['R']};")
        fpar = k.reg("r")
        k(f"div.u32 {fpar}, {jp}, {e['R']};")
        k(f"and.b32 {fpar}, {fpar}, 1;")
        fa = k.reg("r")
        k(f"mad.lo.u32 {fa}, {ds}, 8, {e['fin']};")
        e["wait"](k, fa, fpar, e["status"], 3, e["fail"])
        k("tcgen05.fence::after_thread_sync;")
        no_rs = k.label("NO_RESCALE")
        k(f"@!{anyw} bra {no_rs};")
        e["rescale_o"](alpha)
        k.mark(no_rs)
        k.mark(skip_w)
        k.comment(f"@trace 15 {j}")
        for c in range(4):
            e["st16"](16 * c, packed[16 * c:16 * c + 16])
        e["p_ready_arrive"]()
        k.comment(f"@trace 7 {j}")
        rsum = e["row_sum"](ps2)
        k(f"fma.rn.f32 {lsum}, {lsum}, {alpha}, {rsum};")
        k(f"add.u32 {j}, {j}, 1;")
        pl3 = k.reg("p")
        k(f"setp.lt.u32 {pl3}, {j}, {e['NB']};")
        k(f"@{pl3} bra {e['top3']};")

    def poly_pairs(self) -> set:
        """Which of the 16 column pairs of a 32-column chunk take the FMA-pipe
        exp2 (``POLY`` of them, spread evenly)."""
        n = self.POLY[self.D] if isinstance(self.POLY, dict) else self.POLY
        return {(2 * i + 1) * 16 // (2 * n) for i in range(n)} if n else set()

    @staticmethod
    def _exp2_poly(k, t2, e0, e1, cst):
        """2^x of an f32 pair on the FMA pipe (Cody-Waite split): x clamped to
        >= -126, n = round(x) by adding 1.5 * 2^23, f = x - n in [-0.5, 0.5],
        2^f by the degree-3 minimax polynomial ``EXP2_POLY`` (relative error
        7.5e-5, below the bf16 rounding of P), then n added to the exponent
        field (n * 2^23 taken from the low bits of x + 1.5 * 2^23)."""
        t0, t1 = k.reg("f"), k.reg("f")
        k(f"mov.b64 {{{t0}, {t1}}}, {t2};")
        k(f"max.f32 {t0}, {t0}, {cst['clamp']};")
        k(f"max.f32 {t1}, {t1}, {cst['clamp']};")
        x2 = k.reg("rd")
        k(f"mov.b64 {x2}, {{{t0}, {t1}}};")
        j2 = k.reg("rd")
        k(f"add.rn.f32x2 {j2}, {x2}, {cst['magic']};")
        n2 = k.reg("rd")
        k(f"sub.rn.f32x2 {n2}, {j2}, {cst['magic']};")
        f2 = k.reg("rd")
        k(f"sub.rn.f32x2 {f2}, {x2}, {n2};")
        p2 = k.reg("rd")
        k(f"fma.rn.f32x2 {p2}, {cst['c3']}, {f2}, {cst['c2']};")
        k(f"fma.rn.f32x2 {p2}, {p2}, {f2}, {cst['c1']};")
        k(f"fma.rn.f32x2 {p2}, {p2}, {f2}, {cst['c0']};")
        jr = k.regs("r", 2)
        k(f"mov.b64 {{{jr[0]}, {jr[1]}}}, {j2};")
        pr = k.regs("r", 2)
        k(f"mov.b64 {{{pr[0]}, {pr[1]}}}, {p2};")
        for e, a, b in ((e0, jr[0], pr[0]), (e1, jr[1], pr[1])):
            r = k.reg("r")
            k(f"mad.lo.u32 {r}, {a}, 8388608, {b};")
            k(f"mov.b32 {e}, {r};")

    @staticmethod
    def _scale_pairs(k, regs, s2):
        """regs[i] *= s for 32 f32 registers, as 16 f32x2 multiplies."""
        for i in range(0, len(regs), 2):
            x2 = k.reg("rd")
            k(f"mov.b64 {x2}, {{{regs[i]}, {regs[i + 1]}}};")
            k(f"mul.rn.f32x2 {x2}, {x2}, {s2};")
            k(f"mov.b64 {{{regs[i]}, {regs[i + 1]}}}, {x2};")

    @staticmethod
    def _zero(k):
        r = k.reg("r")
        k(f"mov.u32 {r}, 0;")
        return r


def _bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(v)))[0]


def _f32hex(v: float) -> str:
    return "%08X" % _bits(v)

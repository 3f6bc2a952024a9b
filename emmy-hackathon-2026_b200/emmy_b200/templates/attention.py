"""Attention template: ``O = softmax(Q K^T * s) V`` as a flash-attention kernel
on the 5th-generation tensor cores.

Matches Emmy's attention schedule (reference ``problems/a01_attention``,
``a02_attention_128``: per key ``a1``, a q.k dot-product ``Loop`` per output
row, the online-softmax ``Assign``/``Accum`` chain with the running max
(``acc1``), the running sum (``acc3``) and the weighted sum of V (``acc5``),
then ``reciprocal`` + ``multiply``), here with leading batch/head axes, bf16
Q/K/V [B,H,S,D] and an f32 output.  The reference lowers each thread's
micro-tile to scalar FFMAs that recompute the scores per output column
(``compile.py:1882-1928``).  This template keeps the IR's units of work --
(batch, head, BM query rows), BM = 128 * NT with NT = 1 or 2 query tiles of
128 rows -- and its launch (one CTA per unit).  With two tiles the first 148
CTAs (one per SM) run persistent, looping over the units (CTA c: c, c + 148,
...), and every other CTA returns at once; the units of a partial last
round are split by keys over two CTAs each, the later of the two merging
the partials (``unit_schedule``, ``_merge_split``).  A unit's rows:

* TMA loads the NT Q tiles once per unit (their own producer thread, once
  the previous unit's last Q K^T is done) and K and V tiles of 128 keys into
  two separate rings (3 + 2 stages at D=128, 4 + 4 at D=64; 128-byte
  swizzle; one copy per CTA), each fed by its own producer thread; the
  rings and every per-block barrier run on across units (key blocks are
  counted over all of the CTA's units);
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
from .gemm import WAIT_NS, GemmTemplate, _desc_hi, idesc_mma

LOG2E = 1.4426950408889634
SMEM_MAX = 227 * 1024
# 2^f on [-0.5, 0.5]: degree-3 polynomial minimising the maximum relative
# error (linear-programming fit on 4001 points; 7.5e-5), f32 coefficients
EXP2_POLY = (0.9999280571937561, 0.6932608485221863, 0.24261115491390228, 0.05517221987247467)

# warp roles (512 threads): softmax warps 0..4*NT-1, then these
MMA_WARP, PROD_K_WARP, PROD_V_WARP, PROD_Q_WARP = 8, 9, 10, 11
WORKERS = 148                # persistent CTAs: one per SM of a B200
# registers per thread: at launch, and after setmaxnreg for the softmax
# warpgroups and for the rest (2 x 128 x 200 + 2 x 128 x 56 = 512 x 128)
LAUNCH_REGS, SOFT_REGS, ROLE_REGS = 128, 200, 56


def unit_schedule(units: int, workers: int, split_tail: bool):
    """(W, NF, R, half) of a persistent launch over ``units`` (batch, head,
    256-row query block) units: ``W`` worker CTAs, each runs ``NF`` full
    rounds (CTA c: units c, c + W, ...); ``R`` units are left over.  With
    ``half`` (2R <= W) each leftover unit is split by keys: CTAs 2i and
    2i+1 both compute all 256 rows of leftover unit i, over the first and
    the second half of the key blocks, and the later of the two to finish
    merges the partial results, so the last round costs about half a round;
    otherwise CTAs 0 .. R-1 take one more whole unit."""
    W = min(workers, units)
    NF, R = divmod(units, W)
    return W, NF, R, bool(split_tail and R and 2 * R <= W)


def cta_units(c: int, units: int, workers: int, split_tail: bool):
    """The work list of CTA ``c``: (unit, key half: None for all keys, else 0
    or 1) per iteration -- the order every role walks."""
    W, NF, R, half = unit_schedule(units, workers, split_tail)
    out = [(c + W * i, None) for i in range(NF)] if c < W else []
    if c < W and half and c < 2 * R:
        out.append((NF * W + c // 2, c % 2))
    elif c < W and not half and c < R:
        out.append((NF * W + c, None))
    return out


def unit_rows(k, u, cta, sched, QB, S, NT, want_q=True):
    """Emitted form of ``cta_units``: unit iteration ``u`` of CTA ``cta`` ->
    registers (first query row, first key row) of its unit in the flattened
    [B*H*S] row space, and the split-unit predicate (None without a split
    tail; the key row then already starts at the CTA's half of the keys)."""
    W, NF, _, half = sched
    uu = k.reg("r")
    k(f"mad.lo.u32 {uu}, {u}, {W}, {cta};")
    ph_ = None
    if half:                       # unit NF*W + cta/2, rows 128*(cta%2) of it
        ph_ = k.reg("p")
        k(f"setp.ge.u32 {ph_}, {u}, {NF};")
        tl = k.reg("r")
        k(f"shr.u32 {tl}, {cta}, 1;")
        k(f"add.u32 {tl}, {tl}, {NF * W};")
        k(f"selp.u32 {uu}, {tl}, {uu}, {ph_};")
    bh = k.reg("r")
    k(f"div.u32 {bh}, {uu}, {QB};")
    krow0 = k.reg("r")
    k(f"mul.lo.u32 {krow0}, {bh}, {S};")
    qrow0 = None
    if want_q:
        qb = k.reg("r")
        k(f"rem.u32 {qb}, {uu}, {QB};")
        qrow0 = k.reg("r")
        k(f"mad.lo.u32 {qrow0}, {qb}, {128 * NT}, {krow0};")
    if half:                       # this CTA's half of the keys
        hs = k.reg("r")
        k(f"and.b32 {hs}, {cta}, 1;")
        k(f"mul.lo.u32 {hs}, {hs}, {S // 2};")
        k(f"selp.u32 {hs}, {hs}, 0, {ph_};")
        k(f"add.u32 {krow0}, {krow0}, {hs};")
    return qrow0, krow0, ph_


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
    # (3,200 cycles a pass instead of 1,750), a 4,570-cycle block period.
    # At D = 64 pairs run the split-P form (each CTA 32 columns of every V
    # block in 64-byte swizzled boxes; S_FREE and P_READY count both CTAs'
    # softmax warps): correct, and slower too (557 against 743 TFLOP/s)
    PAIR = {64: False, 128: False}
    # two-tile CTAs run persistent: the first WORKERS CTAs loop over the
    # (batch, head, 256-row) units and every other CTA returns at once; with
    # TAIL_SPLIT the units of a partial last round are split by keys over
    # two CTAs each
    PERSIST = True
    TAIL_SPLIT = True

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
        if ctx.block != (512, 1, 1) or tuple(ctx.grid[1:]) != (1, 1) or \
                ctx.grid[0] != B * H * S // BM:
            raise TemplateMismatch("launch geometry (512 threads, a 1-D grid of one CTA per unit)")
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
        # (a CTA's half of a V block is D/2 columns: whole 64-column boxes)
        self.pair = (bool(cls.PAIR.get(D, False)) and self.NT == 2
                     and D % 64 == 0 and (S // 256) % 2 == 0 and tuple(ctx.grid[1:]) == (1, 1))
        if self.pair:
            # K and V stages hold half a block each: twice as many fit
            n = min(12, avail // (TB // 2))
            self.SK, self.SV = (n + 1) // 2, n // 2
        self.units = B * H * S // BM
        # persistent only when the launch's shared memory keeps one CTA per
        # SM (228 KiB an SM): two co-resident workers would queue on the
        # 512-column tensor-memory allocation while other SMs sit idle
        self.persist = (bool(cls.PERSIST) and self.NT == 2 and not self.pair
                        and ctx.smem_bytes > 114 * 1024)
        self.sched = unit_schedule(self.units, WORKERS if self.persist else self.units,
                                   self.persist and bool(cls.TAIL_SPLIT))
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
        W_, _, RU_, half_ = self.sched
        if half_:
            # split units: each CTA's partial O [256][D], then its m[256]
            # and l[256], per (leftover unit, key half); one arrival counter
            # per leftover unit, 2 added per launch (even: nobody finished)
            k.decl(f".global .align 32 .b8 __emmy_part[{2 * RU_ * 256 * (D + 2) * 4}];")
            k.decl(f".global .align 4 .u32 __emmy_pairs[{RU_}];")
        rows = self.B * self.H * S
        # a pair's V half is D/2 columns: 64-column boxes (128-byte rows,
        # 128-byte swizzle), or at D = 64 one 32-column box (64-byte rows,
        # 64-byte swizzle)
        VBOX = min(64, D // 2) if pair else 64
        for nm, buf in (("tmapQ", self.q), ("tmapK", self.k), ("tmapV", self.v)):
            bk = 64 if pair and nm == "tmapK" else 128
            bw, sw = (VBOX, 3 if VBOX == 64 else 2) if nm == "tmapV" else (64, 3)
            k.directive(f"tmap {nm} buf={buf} dtype=9 dims={D},{rows} strides={D * 2} "
                        f"box={bw},{bk} swizzle={sw}")
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
        W, NF, RU, half = self.sched
        if W < self.units or half:
            k.comment(f"persistent: {W} worker CTAs, {NF} full rounds of {self.units} units"
                      + (f", {RU} leftover units split by keys over {2 * RU} CTAs" if half
                         else f", {RU} leftover units"))
        pidle = k.reg("p")
        k(f"setp.ge.u32 {pidle}, {cta}, {W};")
        idle = k.label("IDLE")
        k(f"@{pidle} bra {idle};")
        nunit = k.reg("r")                 # units of this CTA
        pnu = k.reg("p")
        k(f"setp.lt.u32 {pnu}, {cta}, {2 * RU if half else RU};")
        k(f"selp.u32 {nunit}, {NF + 1}, {NF}, {pnu};")
        u = k.reg("r")                     # unit iteration of the role
        g0 = k.reg("r")                    # its first key block, counted over all units
        gend = k.reg("r")                  # one past its last

        def unit_coords(want_q=True):
            """(first query row, first key row, half-unit predicate or None) of
            unit iteration ``u``; sets ``g0`` and ``gend``."""
            k(f"mul.lo.u32 {g0}, {u}, {NB};")
            k(f"add.u32 {gend}, {g0}, {NB};")
            r = unit_rows(k, u, cta, self.sched, QB, S, NT, want_q)
            if half:                       # a split unit: half of the key blocks
                k(f"@{r[2]} sub.u32 {gend}, {gend}, {NB // 2};")
            return r

        def unit_loop_tail(top):
            k(f"add.u32 {u}, {u}, 1;")
            pu = k.reg("p")
            k(f"setp.lt.u32 {pu}, {u}, {nunit};")
            k(f"@{pu} bra {top};")
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
        Q_EMPTY = DRAIN + 1            # every Q K^T of the unit done: Q may be reloaded
        MERGE_READY = Q_EMPTY + 1      # split unit: every softmax warp wrote its partial
        MERGE_GO = MERGE_READY + 1     # split unit: this CTA merges
        MERGE_SKIP = MERGE_GO + 1      # split unit: the other CTA merges
        NSLOT = MERGE_SKIP + 1
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
                # pair: the leader's counts both CTAs' softmax warps
                cnt = (8 if pair else 4) * NT if slot in (P_READY, S_FREE) else 1
            else:
                # pair: the leader's P_READY counts both CTAs' softmax warps
                cnt = (8 if pair else 4) if P_READY <= slot < P_READY + NT else 1
            if slot == MERGE_READY:
                cnt = 4 * NT
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

        # the leader's waits on barriers the peer CTA's warps arrive on
        csem = ".acquire.cluster" if pair else ""
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

        def producer(which, warp_id, tmap, ring=None, depth=0, full=None, empty=None):
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
            k(f"mov.u32 {u}, 0;")
            utop = k.label(f"UNIT_{which}")
            k.mark(utop)
            if which == "Q":
                # the unit's Q tiles, once the previous unit's last Q K^T is done
                qrow0, _, _ = unit_coords()
                first = k.label("Q_FIRST")
                pu0 = k.reg("p")
                k(f"setp.eq.u32 {pu0}, {u}, 0;")
                k(f"@{pu0} bra {first};")
                qpar = k.reg("r")
                k(f"sub.u32 {qpar}, {u}, 1;")
                k(f"and.b32 {qpar}, {qpar}, 1;")
                wait(k, bar(Q_EMPTY), qpar, status, 1, end_p)
                k.mark(first)
                qf = bar(Q_FULL)
                k(f"{arm}mbarrier.arrive.expect_tx.shared::cta.b64 _, [{qf}], {ncta * NT * TB};")
                qft = target(qf)
                for t in range(NT):
                    qr = k.reg("r")
                    k(f"add.u32 {qr}, {qrow0}, {128 * t};")
                    for i in range(NBX):
                        k(f"{cpy} [{qs}+{t * TB + i * 16384}], [{tq}, {{{64 * i}, {qr}}}], "
                          f"[{qft}];")
                unit_loop_tail(utop)
                k.mark(end_p)
                return
            _, krow0, _ = unit_coords(want_q=False)
            k(f"mov.u32 {j}, {g0};")       # j counts key blocks over all units
            top = k.label(f"PROD_{which}")
            k.mark(top)
            st_, ph_ = ring_slot(j, depth)
            if split:
                # the stage's previous block b = j - depth is free once the
                # P V iteration that last read it is done: V(b) -> DONE(b);
                # K(b), read by the Q K^T issued in iteration b-1 -> DONE(b-1),
                # or, the first block of a unit (its Q K^T issued before the
                # unit's first iteration) -> DONE(b)
                nowait = k.label(f"NOWAIT_{which}")
                pf = k.reg("p")
                k(f"setp.lt.u32 {pf}, {j}, {depth};")
                k(f"@{pf} bra {nowait};")
                n_ = k.reg("r")
                k(f"sub.u32 {n_}, {j}, {depth};")
                if which == "K":
                    bm = k.reg("r")
                    k(f"rem.u32 {bm}, {n_}, {NB};")
                    pb = k.reg("p")
                    k(f"setp.ne.u32 {pb}, {bm}, 0;")
                    k(f"@{pb} sub.u32 {n_}, {n_}, 1;")
                ds, dph = ring_slot(n_, R)
                wait(k, bar(DONE, ds), dph, status, 1, end_p)
                k.mark(nowait)
            else:
                par = k.reg("r")
                k(f"xor.b32 {par}, {ph_}, 1;")
                wait(k, bar(empty, st_), par, status, 1, end_p)
            kr = k.reg("r")
            k(f"sub.u32 {kr}, {j}, {g0};")
            k(f"mad.lo.u32 {kr}, {kr}, 128, {krow0};")
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
                for i in range((D // 2) // VBOX):
                    ci = k.reg("r")
                    k(f"add.u32 {ci}, {c0}, {VBOX * i};")
                    k(f"{cpy} [{dst}+{i * 128 * VBOX * 2}], [{tmap}, {{{ci}, {kr}}}], [{fbt}];")
            else:
                for i in range(NBX):
                    k(f"{cpy} [{dst}+{i * 16384}], [{tmap}, {{{64 * i}, {kr}}}], [{fbt}];")
            k.comment(f"@trace {10 if which == 'K' else 11} {j}")
            k(f"add.u32 {j}, {j}, 1;")
            pl = k.reg("p")
            k(f"setp.lt.u32 {pl}, {j}, {gend};")
            k(f"@{pl} bra {top};")
            unit_loop_tail(utop)
            k.mark(end_p)

        # ---------------- producers: Q, K and V, one warp each ----------------
        producer("Q", PROD_Q_WARP, tq)
        producer("K", PROD_K_WARP, tk, kring, SK, K_FULL, K_EMPTY)
        producer("V", PROD_V_WARP, tv, vring, SV, V_FULL, V_EMPTY)

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
        # V: MN-major, 128 keys x VBOX columns a box; 16 key rows a K step
        VROW = VBOX * 2                               # bytes of a V box row
        hiV = (_desc_hi(16384, 1024) if VROW == 128 else
               _desc_hi(128 * VROW, 8 * VROW, 4))     # 64-byte swizzle (layout 4)
        ptrue = k.reg("p")
        k(f"setp.eq.u32 {ptrue}, 0, 0;")
        pfalse = k.reg("p")
        k(f"setp.ne.u32 {pfalse}, 0, 0;")
        zero = k.reg("r")
        k(f"mov.u32 {zero}, 0;")
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
                k(f"add.s64 {bd}, {dv}, {kk * VROW};")  # +16 key rows (16-byte units)
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
        k(f"mov.u32 {u}, 0;")
        mtop = k.label("UNIT_M")
        k.mark(mtop)
        unit_coords(want_q=False)
        glast = k.reg("r")
        k(f"sub.u32 {glast}, {gend}, 1;")
        qpar = k.reg("r")
        k(f"and.b32 {qpar}, {u}, 1;")
        wait(k, bar(Q_FULL), qpar, status, 2, end_mma)
        # block 0 scores of every tile
        k(f"mov.u32 {j}, {g0};")
        dk0, kst0 = k_ready(j)
        if split:
            # the previous unit's last scores have been read
            sfirst = k.label("S_FIRST")
            pu0 = k.reg("p")
            k(f"setp.eq.u32 {pu0}, {u}, 0;")
            k(f"@{pu0} bra {sfirst};")
            spar0 = k.reg("r")
            k(f"sub.u32 {spar0}, {j}, 1;")
            k(f"and.b32 {spar0}, {spar0}, 1;")
            wait(k, bar(S_FREE), spar0, status, 2, end_mma, csem)
            k("tcgen05.fence::after_thread_sync;")
            k.mark(sfirst)
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
            k(f"setp.ne.u32 {pacc}, {j}, {g0};")
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
                wait(k, bar(S_FREE), par, status, 2, end_mma, csem)
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
            k(f"setp.ne.u32 {pacc}, {j}, {g0};")
            wait(k, bar(P_READY), par, status, 2, end_mma, csem)
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
            k(f"setp.lt.u32 {pl2}, {j}, {glast};")
            k(f"@{pl2} bra {top2};")
        # every Q K^T of the unit is issued: Q is free once they complete
        commit(bar(Q_EMPTY))
        k(f"mov.u32 {j}, {glast};")
        block(True)
        unit_loop_tail(mtop)
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
        units_done = k.label("UNITS_DONE")
        k(f"mov.u32 {u}, 0;")
        stop = k.label("UNIT_S")
        k.mark(stop)
        qrow0, _, shalf = unit_coords()
        m = k.reg("f")                             # max used for the exponents
        k(f"mov.f32 {m}, 0fFF800000;")
        lsum = k.reg("f")
        k(f"mov.f32 {lsum}, 0f00000000;")
        k(f"mov.u32 {j}, {g0};")
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

        lsfree = None
        if pair:
            # the P_READY (and, with split P, S_FREE) the leader's issuing
            # thread waits on
            lpready = k.reg("r")
            k(f"mapa.shared::cluster.u32 {lpready}, {pready}, 0;")
            if split:
                lsfree = k.reg("r")
                k(f"mapa.shared::cluster.u32 {lsfree}, {sfree}, 0;")

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
                lsfree=lsfree,
                fin=fin, pl0=pl0, g0=g0, gend=gend, R=R, status=status, fail=soft_teardown,
                wait=wait))
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
            k(f"setp.eq.u32 {pj0}, {j}, {g0};")
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
            k(f"setp.lt.u32 {pl3}, {j}, {gend};")
            k(f"@{pl3} bra {top3};")
        # epilogue: O row * (1 / l) -> global
        def done_wait(blk):
            """Wait for DONE of key block ``blk`` (a register): ring slot
            blk % R, its (blk / R)-th completion."""
            ds = k.reg("r")
            k(f"rem.u32 {ds}, {blk}, {R};")
            fpar = k.reg("r")
            k(f"div.u32 {fpar}, {blk}, {R};")
            k(f"and.b32 {fpar}, {fpar}, 1;")
            fa = k.reg("r")
            k(f"mad.lo.u32 {fa}, {ds}, 8, {fin};")
            wait(k, fa, fpar, status, 3, soft_teardown)

        if split:
            # the unit's last block's P V
            gl = k.reg("r")
            k(f"sub.u32 {gl}, {gend}, 1;")
            done_wait(gl)
        else:
            fpar = k.reg("r")                      # FINAL completes once per unit
            k(f"and.b32 {fpar}, {u}, 1;")
            wait(k, fin, fpar, status, 3, soft_teardown)
        k("tcgen05.fence::after_thread_sync;")
        if half:
            merge = k.label("MERGE")
            k(f"@{shalf} bra {merge};")
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
        unit_loop_tail(stop)
        if half:
            k(f"bra {units_done};")
            k.mark(merge)
            self._merge_split(k, dict(
                cta=cta, tid=tid, tt=tt, row=row, orow_tm=orow_tm, m=m, lsum=lsum, qrow0=qrow0,
                obase=obase, wait_ld=wait_ld, done=units_done, pl0=pl0,
                ready=bar(MERGE_READY), go=bar(MERGE_GO), skip=bar(MERGE_SKIP), status=status,
                fail=soft_teardown, wait=wait))
        k.mark(units_done)
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
        k.mark(idle)
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
        if e.get("lsfree"):
            # a pair: on the leader's S_FREE, released to the cluster
            k(f"@{e['pl0']} mbarrier.arrive.release.cluster.shared::cluster.b64 _, "
              f"[{e['lsfree']}];")
        else:
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
        k(f"setp.eq.u32 {pj0}, {j}, {e['g0']};")
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
        k(f"setp.lt.u32 {pl3}, {j}, {e['gend']};")
        k(f"@{pl3} bra {e['top3']};")

    def _merge_split(self, k, e):
        """Epilogue of a key-split unit.  CTAs 2i and 2i+1 each hold all 256
        rows of leftover unit i over one half of the keys.  Every softmax
        thread writes its row's partial -- O unnormalised (to the row's base
        m), m and l -- to ``__emmy_part`` and fences it (gpu scope); once all
        softmax warps have arrived on MERGE_READY, thread 0 adds 1 to the
        unit's counter (acq_rel, gpu scope) and publishes the old value
        through shared memory (MERGE_GO).  Old value even: the other CTA has
        not finished and will merge; this CTA is done.  Odd: the other's
        partial is complete and each thread merges its row.  Thread 0 tells
        the others by which barrier it arrives on (MERGE_GO or MERGE_SKIP;
        they poll both, bounded like every wait):
        m = max(m_a, m_b), f = 2^(m_x - m), l = l_a f_a + l_b f_b,
        O = (O_a f_a + O_b f_b) / l -- a product per side and one add, so
        the result does not depend on which CTA merges.  No thread waits for
        the other CTA: the later one merges, whichever it is.  The scratch
        and the counters belong to the module, so two launches of one module
        must not overlap in time (launches on one stream never do)."""
        D = self.D
        W, _, RU, _ = self.sched
        PER = 256 * (D + 2) * 4                 # bytes per (unit, key half)
        cta, tt, row = e["cta"], e["tt"], e["row"]
        slot = k.reg("r")
        k(f"shr.u32 {slot}, {cta}, 1;")
        hk = k.reg("r")
        k(f"and.b32 {hk}, {cta}, 1;")
        rr = k.reg("r")                         # row within the unit
        k(f"mad.lo.u32 {rr}, {tt}, 128, {row};")
        part = k.reg("rd")
        k(f"mov.u64 {part}, __emmy_part;")

        def rows_of(half_reg):
            """(O row, m, l) addresses of row rr in the partial of key half
            ``half_reg``."""
            pi = k.reg("r")
            k(f"mad.lo.u32 {pi}, {slot}, 2, {half_reg};")
            base = k.reg("rd")
            k(f"mul.wide.u32 {base}, {pi}, {PER};")
            k(f"add.s64 {base}, {base}, {part};")
            o = k.reg("rd")
            k(f"mul.wide.u32 {o}, {rr}, {D * 4};")
            k(f"add.s64 {o}, {o}, {base};")
            ml = k.reg("rd")
            k(f"mul.wide.u32 {ml}, {rr}, 4;")
            k(f"add.s64 {ml}, {ml}, {base};")
            return o, ml                        # m at ml + 256 D 4, l 1 KiB after

        own_o, own_ml = rows_of(hk)
        for c in range(D // 32):
            regs = k.regs("r", 32)
            k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, "
              f"[{e['orow_tm']}+{32 * c}];")
            e["wait_ld"]()
            for v8 in range(4):
                k(f"st.global.v8.b32 [{own_o}+{128 * c + 32 * v8}], "
                  f"{{{', '.join(regs[8 * v8:8 * v8 + 8])}}};")
        k(f"st.global.f32 [{own_ml}+{256 * D * 4}], {e['m']};")
        k(f"st.global.f32 [{own_ml}+{256 * (D + 1) * 4}], {e['lsum']};")
        k("fence.acq_rel.gpu;")
        k("bar.warp.sync 0xffffffff;")
        k(f"@{e['pl0']} mbarrier.arrive.shared::cta.b64 _, [{e['ready']}];")
        pt0 = k.reg("p")
        k(f"setp.eq.u32 {pt0}, {e['tid']}, 0;")
        not0 = k.label("MERGE_WAIT")
        k(f"@!{pt0} bra {not0};")
        e["wait"](k, e["ready"], 0, e["status"], 3, e["fail"])
        cnt = k.reg("rd")
        k(f"mov.u64 {cnt}, __emmy_pairs;")
        ca = k.reg("rd")
        k(f"mul.wide.u32 {ca}, {slot}, 4;")
        k(f"add.s64 {ca}, {ca}, {cnt};")
        old = k.reg("r")
        k(f"atom.acq_rel.gpu.global.add.u32 {old}, [{ca}], 1;")
        k(f"and.b32 {old}, {old}, 1;")
        psecond = k.reg("p")
        k(f"setp.ne.u32 {psecond}, {old}, 0;")
        k(f"@{psecond} mbarrier.arrive.shared::cta.b64 _, [{e['go']}];")
        k(f"@!{psecond} mbarrier.arrive.shared::cta.b64 _, [{e['skip']}];")
        k.mark(not0)
        # poll both decisions, bounded by %globaltimer
        domerge = k.label("MERGE_ROWS")
        pg, ps = k.reg("p"), k.reg("p")
        t0, t1 = k.reg("rd"), k.reg("rd")
        k(f"mov.u64 {t0}, %globaltimer;")
        poll = k.label("MERGE_POLL")
        k.mark(poll)
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {pg}, [{e['go']}], 0;")
        k(f"@{pg} bra {domerge};")
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {ps}, [{e['skip']}], 0;")
        k(f"@{ps} bra {e['done']};")
        k(f"mov.u64 {t1}, %globaltimer;")
        k(f"sub.s64 {t1}, {t1}, {t0};")
        pt = k.reg("p")
        k(f"setp.lt.s64 {pt}, {t1}, {WAIT_NS};")
        k(f"@{pt} bra {poll};")
        k(f"st.global.u32 [{e['status']}], 3;")
        k(f"bra {e['fail']};")
        k.mark(domerge)
        # the other CTA's partial is complete: merge
        k("fence.acq_rel.gpu;")
        ho = k.reg("r")
        k(f"xor.b32 {ho}, {hk}, 1;")
        oth_o, oth_ml = rows_of(ho)
        mb, lb = k.reg("f"), k.reg("f")
        k(f"ld.global.f32 {mb}, [{oth_ml}+{256 * D * 4}];")
        k(f"ld.global.f32 {lb}, [{oth_ml}+{256 * (D + 1) * 4}];")
        mm = k.reg("f")
        k(f"max.f32 {mm}, {e['m']}, {mb};")
        fa, fb, t_ = k.reg("f"), k.reg("f"), k.reg("f")
        k(f"sub.rn.f32 {t_}, {e['m']}, {mm};")
        k(f"ex2.approx.ftz.f32 {fa}, {t_};")
        k(f"sub.rn.f32 {t_}, {mb}, {mm};")
        k(f"ex2.approx.ftz.f32 {fb}, {t_};")
        la, l_ = k.reg("f"), k.reg("f")
        k(f"mul.rn.f32 {la}, {e['lsum']}, {fa};")
        k(f"mul.rn.f32 {l_}, {lb}, {fb};")
        k(f"add.rn.f32 {l_}, {la}, {l_};")
        inv = k.reg("f")
        k(f"rcp.rn.f32 {inv}, {l_};")
        grow = k.reg("r")
        k(f"add.u32 {grow}, {rr}, {e['qrow0']};")
        oa = k.reg("rd")
        k(f"mul.wide.u32 {oa}, {grow}, {D * 4};")
        k(f"add.s64 {oa}, {oa}, {e['obase']};")
        for c in range(D // 32):
            regs = k.regs("r", 32)
            k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, "
              f"[{e['orow_tm']}+{32 * c}];")
            e["wait_ld"]()
            for v4 in range(8):
                ob = k.regs("f", 4)
                k(f"ld.global.v4.f32 {{{', '.join(ob)}}}, [{oth_o}+{128 * c + 16 * v4}];")
                for i in range(4):
                    a = regs[4 * v4 + i]
                    x = k.reg("f")
                    k(f"mul.rn.f32 {x}, {a}, {fa};")
                    y = k.reg("f")
                    k(f"mul.rn.f32 {y}, {ob[i]}, {fb};")
                    k(f"add.rn.f32 {x}, {x}, {y};")
                    k(f"mul.rn.f32 {x}, {x}, {inv};")
                    k(f"mov.b32 {a}, {x};")
            for v8 in range(4):
                k(f"st.global.v8.b32 [{oa}+{128 * c + 32 * v8}], "
                  f"{{{', '.join(regs[8 * v8:8 * v8 + 8])}}};")

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

"""bf16 matmul on persistent CTA pairs with a double-buffered accumulator.

The IR launches one CTA per 128 x 256 output tile; when its shared-memory
budget allows a deep ring (at least 4 pair stages, so one CTA per SM), the
first ``WORKERS`` clusters of 2 CTAs (one per SM pair of the B200's 148 SMs)
do all the work and every other cluster returns at once (measured: 3,948
such CTAs cost about 6 us in total).  Cluster c computes the 256 x 256 pair
tiles ``c, c + WORKERS, c + 2*WORKERS, ...`` -- tiles are numbered down
groups of ``GROUP_M`` 256-row bands, column block by column block, so the
tiles in flight share a few A bands and B panels in L2 -- exactly the CTA-pair scheme of ``gemm_pair``
(leader-issued ``tcgen05.mma.cta_group::2``, each CTA loading its A rows and
half of B, both CTAs' copies completing on the leader's ``full`` barrier),
with three changes:

* the shared-memory ring runs continuously across tiles: the producer
  starts the next tile's k-slices while the MMA thread finishes the current
  one;
* tensor memory holds two 256-column accumulators (all 512 columns): tile i
  accumulates into buffer ``i % 2``;
* warps 4-7 of both CTAs are the epilogue: they wait for the tile's ``acc``
  barrier, drain their 32 rows x 256 columns (``tcgen05.ld.32x32b.x32``,
  32-byte stores), then arrive on the leader's ``acc_empty`` barrier for that
  buffer (8 arrivals: 4 warps x 2 CTAs, the follower's through ``mapa``),
  which the MMA thread waits on before reusing the buffer -- so each CTA's
  epilogue overlaps its own next main loop.

Warp 0 lane 0 is the producer, warp 1 allocates tensor memory and its lane
0 in the leader issues the MMAs; warps 2-3 join the conversion in 3xTF32
mode (six converter warps per CTA) and otherwise only the teardown.  Every
mbarrier wait is bounded by ``%globaltimer`` (codes 1 producer, 2 MMA issuer,
3 epilogue, 6 accumulator reuse); a role whose wait expires leaves its loop.
"""
from __future__ import annotations

from ..ptx import Kernel
from . import gemm as _gemm
from .gemm import GemmTemplate, _desc_hi, idesc_mma, tf32_lo_trunc, tf32_split

WORKERS = 74                 # clusters of 2 CTAs: the 148 SMs of a B200
PERSISTENT_MIN_STAGES = 4    # 4 x 32 KiB ring: one CTA per SM
EPI_CHUNK = 16               # accumulator columns per tcgen05.ld in the epilogue
GROUP_M = 16                 # 256-row bands per raster group (tiles run down a group's bands)
# 3xTF32 operands are twice as wide: 8 bands a group read 1.12 GB from DRAM at
# M=N=8192, K=4096 against 1.27 GB with 16 and 1.45 GB with 4 (ncu, same
# call), at 278.7 / 278.4 / 274.4 TFLOP/s on the BASELINE shape
GROUP_M_TF32 = 8
TAIL_SPLIT = True            # leftover pair tiles of a partial last round run as 256 x 128 halves
# 3xTF32: the A operand's raw (high) and low parts in tensor memory instead of
# shared memory (tcgen05.mma's [a-tmem] form), one accumulator instead of two.
# Measured on one B200 (same process, alternating, outputs checked): M=16384
# 268.1-268.5 -> 275.1-275.4 TFLOP/s, M=4096 269.7-270.1 -> 277.6-277.7,
# M=2048 (one GPU's shard at 8 GPUs) 239.6 -> 250.7-251.3
TF32_A_TMEM = True


def schedule(tiles: int, workers: int = WORKERS):
    """(W, NF, R, half): ``W`` worker clusters; every cluster runs ``NF``
    full rounds of 256 x 256 pair tiles (cluster c: tiles c, c + W, ...);
    ``R`` tiles are left over.  With ``half``, the leftover tiles are cut
    into 256 x 128 halves and clusters 0 .. 2R-1 take one half each, so the
    last round costs about half a round instead of a whole one (256 tiles
    on 74 clusters: 3.5 rounds, not 4).  Without it (2R above W, where the
    halves would need two half rounds anyway) clusters 0 .. R-1 take one
    more whole tile."""
    W = min(workers, tiles)
    NF, R = divmod(tiles, W)
    return W, NF, R, bool(TAIL_SPLIT and R and 2 * R <= W)


def cluster_tiles(c: int, tiles: int, workers: int = WORKERS):
    """The work list of cluster ``c`` under ``schedule``: (pair tile index
    in raster order, column offset 0 or 128, width 256 or 128) per
    iteration -- the order the kernel's producer, MMA and epilogue roles
    walk."""
    W, NF, R, half = schedule(tiles, workers)
    out = [(c + W * i, 0, 256) for i in range(NF)]
    if half:
        if c < 2 * R:
            out.append((NF * W + c // 2, 128 * (c % 2), 128))
    elif c < R:
        out.append((c + W * NF, 0, 256))
    return out


def tile_index(k, idx, clus, W, NF, half):
    """Emitted form of ``cluster_tiles``: iteration ``idx`` of cluster
    ``clus`` -> (pair tile register in raster order, half-tile predicate or
    None, column offset register or None: 128 on the second half)."""
    tt = k.reg("r")
    k(f"mad.lo.u32 {tt}, {idx}, {W}, {clus};")
    if not half:
        return tt, None, None
    ph_ = k.reg("p")
    k(f"setp.ge.u32 {ph_}, {idx}, {NF};")
    tail = k.reg("r")                             # tile NF*W + clus/2, half clus%2
    k(f"shr.u32 {tail}, {clus}, 1;")
    k(f"add.u32 {tail}, {tail}, {NF * W};")
    k(f"selp.u32 {tt}, {tail}, {tt}, {ph_};")
    hoff = k.reg("r")
    k(f"and.b32 {hoff}, {clus}, 1;")
    k(f"shl.b32 {hoff}, {hoff}, 7;")
    k(f"selp.u32 {hoff}, {hoff}, 0, {ph_};")
    return tt, ph_, hoff


def raster(k, tt, MB, NB, group=None):
    """Pair tile index -> (256-row band, 256-column block) registers: tiles
    are numbered down groups of ``group`` bands, one column block after the
    other, so consecutive tiles -- the ones in flight together -- share a
    few A bands and B panels in L2 (measured on the BASELINE matmul: 16
    bands 1561 TFLOP/s, 1 band 1402)."""
    GM = min(GROUP_M if group is None else group, MB)
    mp, nbk = k.reg("r"), k.reg("r")
    if GM <= 1:
        k(f"div.u32 {mp}, {tt}, {NB};")
        k(f"rem.u32 {nbk}, {tt}, {NB};")
        return mp, nbk
    # group g = bands [g*GM, g*GM + gm); inside it tile l -> band g*GM + l % gm,
    # column block l / gm (the last group may hold fewer bands)
    g = k.reg("r")
    k(f"div.u32 {g}, {tt}, {GM * NB};")
    first = k.reg("r")
    k(f"mul.lo.u32 {first}, {g}, {GM};")
    gm = k.reg("r")
    k(f"sub.u32 {gm}, {MB}, {first};")
    k(f"min.u32 {gm}, {gm}, {GM};")
    loc = k.reg("r")
    k(f"mul.lo.u32 {loc}, {g}, {GM * NB};")
    k(f"sub.u32 {loc}, {tt}, {loc};")
    k(f"rem.u32 {mp}, {loc}, {gm};")
    k(f"add.u32 {mp}, {mp}, {first};")
    k(f"div.u32 {nbk}, {loc}, {gm};")
    return mp, nbk


def emit_pair_persistent(t) -> str:
    """bf16 (``kind::f16``) or fp32 through 3xTF32 (``kind::tf32``, the
    operands split into tf32 hi/lo parts in shared memory by warps 4-7)."""
    ctx = t.ctx
    tf32 = t.mode == "tf32x3"
    es = 4 if tf32 else 2
    BM, BN, K = 128, 256, t.K
    BK = 128 // es                   # one 128-byte swizzle row of K per stage
    S = t.pair_S
    KT = K // BK
    SA = BM * BK * es                # own A rows: 16 KiB
    SBH = BK * 128 * es              # own half of B: BK k-rows x 128 columns
    RAW = SA + SBH
    STG = 2 * RAW if tf32 else RAW   # 3xTF32 keeps the low parts after the raw slice
    BOXN = 128 // es                 # B boxes are 128 bytes wide
    KMMA = 32 // es                  # K per tcgen05.mma
    CONVW = 6 if tf32 else 0         # 3xTF32 converter warps: 2..7
    # A in tensor memory (3xTF32): one 256-column accumulator, then per ring
    # stage the A rows' raw values (BK columns) and their low parts (BK more)
    ATM = tf32 and TF32_A_TMEM and BN + S * 2 * BK <= 512
    NACC = 1 if ATM else 2
    ABASE = NACC * BN
    NB = t.NB                        # 256-column tiles per row band
    MB = t.M // 256                  # 256-row bands
    TILES = MB * NB                  # pair tiles
    W, NF, R, HALF = schedule(TILES)
    params = ctx.params() + [("tmapA", ".align 64 .b8", "[128]"),
                             ("tmapB", ".align 64 .b8", "[128]")]
    k = Kernel(ctx.entry, params)
    k.maxntid = (256, 1, 1)
    k.maxnreg = 128                  # one CTA per SM: registers are plentiful
    k.reqnctapercluster = (2, 1, 1)
    k.directive("cluster 2 1 1")
    k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
    k.decl(".global .align 4 .u32 __emmy_status;")
    tm = 7 if tf32 else 9            # CU_TENSOR_MAP_DATA_TYPE_FLOAT32 / BFLOAT16
    k.directive(f"tmap tmapA buf={t.A} dtype={tm} dims={K},{t.M} strides={K * es} "
                f"box={BK},{BM} swizzle=3")
    # MN-major 32-bit operands: the 128-byte swizzle with 32-byte atoms
    k.directive(f"tmap tmapB buf={t.B} dtype={tm} dims={t.N},{K} strides={t.N * es} "
                f"box={BOXN},{BK} swizzle={4 if tf32 else 3}")
    k.comment(f"emmy-b200 template: tcgen05 gemm {t.mode} M={t.M} N={t.N} K={K}, persistent CTA "
              f"pairs ({W} workers, {TILES} pair tiles), stages={S}, 2 accumulators")
    cta = k.special("%ctaid.x")
    clus = k.reg("r")
    k(f"shr.u32 {clus}, {cta}, 1;")
    pidle = k.reg("p")
    k(f"setp.ge.u32 {pidle}, {clus}, {W};")
    idle = k.label("IDLE")
    k(f"@{pidle} bra {idle};")
    cbase = k.param_ptr(t.C)
    ta = k.reg("rd")
    k(f"mov.u64 {ta}, param_tmapA;")
    k(f"cvta.param.u64 {ta}, {ta};")
    tb = k.reg("rd")
    k(f"mov.u64 {tb}, param_tmapB;")
    k(f"cvta.param.u64 {tb}, {tb};")
    tid = k.special("%tid.x")
    warp = k.reg("r")
    k(f"shr.u32 {warp}, {tid}, 5;")
    lane = k.reg("r")
    k(f"and.b32 {lane}, {tid}, 31;")
    rank = k.special("%cluster_ctarank")
    plead = k.reg("p")
    k(f"setp.eq.u32 {plead}, {rank}, 0;")
    # this cluster's tile count: NF full rounds, then one leftover tile (or
    # one half of one) for the first clusters
    ntile = k.reg("r")
    ptl = k.reg("p")
    k(f"setp.lt.u32 {ptl}, {clus}, {2 * R if HALF else R};")
    k(f"selp.u32 {ntile}, {NF + 1}, {NF}, {ptl};")
    # shared memory: S stages, then the mbarriers full[S], empty[S],
    # conv[S] (3xTF32, used in the leader), acc[2], acc_empty[2] (leader),
    # and the tensor-memory slot
    NBAR = 3 * S if tf32 else 2 * S
    raw = k.reg("r")
    k(f"mov.u32 {raw}, __emmy_smem;")
    ring = k.reg("r")
    k(f"add.u32 {ring}, {raw}, 1023;")
    k(f"and.b32 {ring}, {ring}, -1024;")
    bars = k.reg("r")
    k(f"add.u32 {bars}, {ring}, {S * STG};")
    accb = k.reg("r")                          # acc[2]
    k(f"add.u32 {accb}, {bars}, {8 * NBAR};")
    acce = k.reg("r")                          # acc_empty[2]
    k(f"add.u32 {acce}, {accb}, 16;")
    tslot = k.reg("r")
    k(f"add.u32 {tslot}, {accb}, 32;")
    status = k.reg("rd")
    k(f"mov.u64 {status}, __emmy_status;")
    p0 = k.reg("p")
    k(f"setp.eq.u32 {p0}, {tid}, 0;")
    skip_init = k.label("SKIP_INIT")
    k(f"@!{p0} bra {skip_init};")
    for s in range(2 * S):
        k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], 1;")
    for s in range(2 * S, NBAR):               # conv[s]: the converter warps of 2 CTAs
        k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], {2 * CONVW};")
    for b in range(NACC):
        k(f"mbarrier.init.shared::cta.b64 [{accb}+{8 * b}], 1;")
        k(f"mbarrier.init.shared::cta.b64 [{acce}+{8 * b}], 8;")
    k("fence.mbarrier_init.release.cluster;")
    k(f"prefetch.tensormap [{ta}];")
    k(f"prefetch.tensormap [{tb}];")
    k.mark(skip_init)
    pw1 = k.reg("p")
    k(f"setp.eq.u32 {pw1}, {warp}, 1;")
    skip_alloc = k.label("SKIP_ALLOC")
    k(f"@!{pw1} bra {skip_alloc};")
    k(f"tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [{tslot}], 512;")
    k("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;")
    k.mark(skip_alloc)
    k("tcgen05.fence::before_thread_sync;")
    k("bar.sync 0;")
    k("barrier.cluster.arrive.release.aligned;")
    k("barrier.cluster.wait.acquire.aligned;")
    k("tcgen05.fence::after_thread_sync;")
    tmem = k.reg("r")
    k(f"ld.shared.u32 {tmem}, [{tslot}];")
    teardown = k.label("TEARDOWN")
    pl0 = k.reg("p")
    k(f"setp.eq.u32 {pl0}, {lane}, 0;")
    it, kt, st, ph = k.reg("r"), k.reg("r"), k.reg("r"), k.reg("r")

    def bar_addr(group, stage_reg):
        r = k.reg("r")
        k(f"mad.lo.u32 {r}, {stage_reg}, 8, {bars};")
        if group:
            k(f"add.u32 {r}, {r}, {8 * S * group};")
        return r

    def stage_base(stage_reg):
        r = k.reg("r")
        k(f"mad.lo.u32 {r}, {stage_reg}, {STG}, {ring};")
        return r

    def half_pred(idx):
        """True on this cluster's 256 x 128 leftover half tile (None when the
        schedule has none)."""
        if not HALF:
            return None
        ph_ = k.reg("p")
        k(f"setp.ge.u32 {ph_}, {idx}, {NF};")
        return ph_

    def tile_coords(idx):
        """(m0 of this CTA, n0 of the pair tile, this CTA's B columns, the
        half-tile predicate) for this cluster's tile iteration ``idx``."""
        tt, ph_, hoff = tile_index(k, idx, clus, W, NF, HALF)
        mp, nbk = raster(k, tt, MB, NB, GROUP_M_TF32 if tf32 else None)
        m0 = k.reg("r")
        k(f"mad.lo.u32 {m0}, {mp}, 2, {rank};")
        k(f"mul.lo.u32 {m0}, {m0}, {BM};")
        n0 = k.reg("r")
        k(f"mul.lo.u32 {n0}, {nbk}, {BN};")
        nh = k.reg("r")
        if HALF:
            k(f"add.u32 {n0}, {n0}, {hoff};")
            wcol = k.reg("r")                     # each CTA holds half of the tile's B
            k(f"selp.u32 {wcol}, 64, 128, {ph_};")
            k(f"mad.lo.u32 {nh}, {rank}, {wcol}, {n0};")
        else:
            k(f"mad.lo.u32 {nh}, {rank}, 128, {n0};")
        return m0, n0, nh, ph_

    def tile_loop_head(label):
        k(f"mov.u32 {it}, 0;")
        top = k.label(label)
        k.mark(top)
        return top

    def tile_loop_tail(top, count=ntile):
        k(f"add.u32 {it}, {it}, 1;")
        pl = k.reg("p")
        k(f"setp.lt.u32 {pl}, {it}, {count};")
        k(f"@{pl} bra {top};")

    def k_loop_tail(top):
        GemmTemplate._advance(k, st, ph, S)
        k(f"add.u32 {kt}, {kt}, 1;")
        pl = k.reg("p")
        k(f"setp.lt.u32 {pl}, {kt}, {KT};")
        k(f"@{pl} bra {top};")

    # ---------------- producer: warp 0, lane 0 of both CTAs ----------------
    # bf16: both CTAs' copies complete on the leader's full barrier, which
    # the leader arms with both CTAs' bytes; 3xTF32: each CTA's converters
    # need to see their own slice land, so copies complete locally
    pprod = k.reg("p")
    k(f"setp.eq.u32 {pprod}, {warp}, 0;")
    k(f"and.pred {pprod}, {pprod}, {pl0};")
    end_prod = k.label("END_PROD")
    k(f"@!{pprod} bra {end_prod};")
    if not tf32:
        lead_full = k.reg("r")
        k(f"mapa.shared::cluster.u32 {lead_full}, {bars}, 0;")
    k(f"mov.u32 {st}, 0;")
    k(f"mov.u32 {ph}, 0;")
    ptop = tile_loop_head("PTILE")
    m0, n0, nh, phalf = tile_coords(it)
    tx = k.reg("r")                               # bytes this CTA's copies deliver
    if HALF:
        k(f"selp.u32 {tx}, {SA + SBH // 2}, {RAW}, {phalf};")
    else:
        k(f"mov.u32 {tx}, {RAW};")
    if not tf32:
        k(f"shl.b32 {tx}, {tx}, 1;")              # the leader arms for both CTAs
    k(f"mov.u32 {kt}, 0;")
    pk = k.label("PK")
    k.mark(pk)
    par = k.reg("r")
    k(f"xor.b32 {par}, {ph}, 1;")
    GemmTemplate._wait(k, bar_addr(1, st), par, status, 1, end_prod)
    own_fb = bar_addr(0, st)
    if tf32:
        fb = own_fb
        k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{own_fb}], {tx};")
        copy = ("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes")
    else:
        fb = k.reg("r")
        k(f"mad.lo.u32 {fb}, {st}, 8, {lead_full};")
        k(f"@{plead} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{own_fb}], {tx};")
        copy = ("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::"
                "complete_tx::bytes")
    kc = k.reg("r")
    k(f"mul.lo.u32 {kc}, {kt}, {BK};")
    da = stage_base(st)
    k(f"{copy} [{da}], [{ta}, {{{kc}, {m0}}}], [{fb}];")
    for i in range(128 // BOXN):
        nx = k.reg("r")
        k(f"add.u32 {nx}, {nh}, {BOXN * i};")
        db = k.reg("r")
        k(f"add.u32 {db}, {da}, {SA + i * BK * 128};")
        guard = f"@!{phalf} " if HALF and i >= 64 // BOXN else ""
        k(f"{guard}{copy} [{db}], [{tb}, {{{nx}, {kc}}}], [{fb}];")
    k_loop_tail(pk)
    tile_loop_tail(ptop)
    k.mark(end_prod)

    # ---------------- MMA issuer: warp 1, lane 0 of the leader ----------------
    pmma = k.reg("p")
    k(f"setp.eq.u32 {pmma}, {warp}, 1;")
    k(f"and.pred {pmma}, {pmma}, {pl0};")
    k(f"and.pred {pmma}, {pmma}, {plead};")
    end_mma = k.label("END_MMA")
    k(f"@!{pmma} bra {end_mma};")
    mask = k.reg("h")
    k(f"mov.b16 {mask}, 3;")
    idesc_full = idesc_mma(2 * BM, BN, True, tf32)
    idesc_half = idesc_mma(2 * BM, BN // 2, True, tf32)
    hiA = _desc_hi(16, 1024)
    hiB = _desc_hi(BK * 128, 512, 1) if tf32 else _desc_hi(BK * 128, 1024)
    k(f"mov.u32 {st}, 0;")
    k(f"mov.u32 {ph}, 0;")
    mtop = tile_loop_head("MTILE")
    idesc = k.reg("r")
    mhalf = half_pred(it)
    if HALF:                                      # N = 128: 64 B columns from each CTA
        k(f"selp.u32 {idesc}, {idesc_half}, {idesc_full}, {mhalf};")
    else:
        k(f"mov.u32 {idesc}, {idesc_full};")
    buf = k.reg("r")
    aph = k.reg("r")                              # use count of this buffer, parity
    if ATM:                                       # one accumulator: tile i is use i
        k(f"mov.u32 {buf}, 0;")
        k(f"and.b32 {aph}, {it}, 1;")
    else:
        k(f"and.b32 {buf}, {it}, 1;")
        k(f"shr.u32 {aph}, {it}, 1;")
        k(f"and.b32 {aph}, {aph}, 1;")
    k(f"xor.b32 {aph}, {aph}, 1;")
    ae = k.reg("r")
    k(f"mad.lo.u32 {ae}, {buf}, 8, {acce};")
    GemmTemplate._wait(k, ae, aph, status, 6, end_mma, sem=".acquire.cluster")
    k("tcgen05.fence::after_thread_sync;")
    dacc = k.reg("r")
    k(f"mad.lo.u32 {dacc}, {buf}, {BN}, {tmem};")
    k(f"mov.u32 {kt}, 0;")
    mk = k.label("MK")
    k.mark(mk)
    if tf32:       # both CTAs' converters have split this stage
        GemmTemplate._wait(k, bar_addr(2, st), ph, status, 2, end_mma, sem=".acquire.cluster")
    else:
        GemmTemplate._wait(k, bar_addr(0, st), ph, status, 2, end_mma)
    k("tcgen05.fence::after_thread_sync;")
    sb = stage_base(st)
    bad = k.reg("r")
    k(f"add.u32 {bad}, {sb}, {SA};")
    adesc = GemmTemplate._desc(k, sb, hiA)
    bdesc = GemmTemplate._desc(k, bad, hiB)
    if tf32:
        lad = k.reg("r")
        k(f"add.u32 {lad}, {sb}, {RAW};")
        lbd = k.reg("r")
        k(f"add.u32 {lbd}, {sb}, {RAW + SA};")
        ldesc_a = GemmTemplate._desc(k, lad, hiA)
        ldesc_b = GemmTemplate._desc(k, lbd, hiB)
    if ATM:
        ahi = k.reg("r")                          # this stage's A columns in TMEM
        k(f"mad.lo.u32 {ahi}, {st}, {2 * BK}, {tmem};")
        k(f"add.u32 {ahi}, {ahi}, {ABASE};")
    pacc = k.reg("p")
    k(f"setp.ne.u32 {pacc}, {kt}, 0;")
    ptrue = k.reg("p")
    k(f"setp.eq.u32 {ptrue}, 0, 0;")
    kind_ = "tf32" if tf32 else "f16"
    first = True
    for kk in range(BK // KMMA):
        ao, bo = kk * 2, kk * KMMA * 8    # +32 B along K (A); +KMMA rows of 128 B (B)
        pairs = [(adesc, bdesc)]
        if tf32:                          # small terms first: lo*hi + hi*lo, then hi*hi
            pairs = [(ldesc_a, bdesc), (adesc, ldesc_b), (adesc, bdesc)]
        if ATM:                           # A from TMEM: KMMA columns a step, low parts BK on
            pairs = [(("t", BK), bdesc), (("t", 0), ldesc_b), (("t", 0), bdesc)]
        for da_, db_ in pairs:
            bd = k.reg("rd")
            k(f"add.s64 {bd}, {db_}, {bo};")
            if isinstance(da_, tuple):
                at = k.reg("r")
                k(f"add.u32 {at}, {ahi}, {da_[1] + kk * KMMA};")
                aop = f"[{at}]"
            else:
                ad = k.reg("rd")
                k(f"add.s64 {ad}, {da_}, {ao};")
                aop = ad
            k(f"tcgen05.mma.cta_group::2.kind::{kind_} [{dacc}], {aop}, {bd}, {idesc}, "
              f"{pacc if first else ptrue};")
            first = False
    k(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      f"[{bar_addr(1, st)}], {mask};")
    k_loop_tail(mk)
    af = k.reg("r")
    k(f"mad.lo.u32 {af}, {buf}, 8, {accb};")
    k(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      f"[{af}], {mask};")
    tile_loop_tail(mtop)
    k.mark(end_mma)

    # -- warps 4-7 of each CTA: epilogue (3xTF32: warps 2-7 convert first) --
    k("bar.warp.sync 0xffffffff;")
    pepi = k.reg("p")
    k(f"setp.ge.u32 {pepi}, {warp}, 4;")
    prole = k.reg("p")
    k(f"setp.ge.u32 {prole}, {warp}, {8 - CONVW if tf32 else 4};")
    k(f"@!{prole} bra {teardown};")
    q = k.reg("r")
    k(f"and.b32 {q}, {warp}, 3;")
    lead_ae = k.reg("r")                          # acc_empty[0] of the leader
    k(f"mapa.shared::cluster.u32 {lead_ae}, {acce}, 0;")
    tl = k.reg("r")
    k(f"shl.b32 {tl}, {q}, 21;")                  # (32*q) << 16: TMEM lane field
    k(f"add.u32 {tl}, {tl}, {tmem};")

    def epilogue(idx):
        ebuf = k.reg("r")
        eph = k.reg("r")
        if ATM:
            k(f"mov.u32 {ebuf}, 0;")
            k(f"and.b32 {eph}, {idx}, 1;")
        else:
            k(f"and.b32 {ebuf}, {idx}, 1;")
            k(f"shr.u32 {eph}, {idx}, 1;")
            k(f"and.b32 {eph}, {eph}, 1;")
        eaf = k.reg("r")
        k(f"mad.lo.u32 {eaf}, {ebuf}, 8, {accb};")
        GemmTemplate._wait(k, eaf, eph, status, 3, teardown)
        k("tcgen05.fence::after_thread_sync;")
        m0e, n0e, _, ehalf = tile_coords(idx)
        row = k.reg("r")
        k(f"mad.lo.u32 {row}, {q}, 32, {lane};")
        k(f"add.u32 {row}, {row}, {m0e};")
        off = k.reg("rd")
        k(f"mul.wide.u32 {off}, {row}, {t.N * 4};")
        c2 = k.reg("rd")
        k(f"mul.wide.u32 {c2}, {n0e}, 4;")
        k(f"add.s64 {off}, {off}, {c2};")
        cptr = k.reg("rd")
        k(f"add.s64 {cptr}, {cbase}, {off};")
        taddr = k.reg("r")
        k(f"mad.lo.u32 {taddr}, {ebuf}, {BN}, {tl};")
        CH = EPI_CHUNK
        skip_half = k.label("EPI_HALF") if HALF else None
        for c in range(BN // CH):
            if HALF and c == BN // 2 // CH:        # a half tile ends at column 128
                k(f"@{ehalf} bra {skip_half};")
            regs = k.regs("r", CH)
            ta2 = k.reg("r")
            k(f"add.u32 {ta2}, {taddr}, {CH * c};")
            k(f"tcgen05.ld.sync.aligned.32x32b.x{CH}.b32 {{{', '.join(regs)}}}, [{ta2}];")
            k("tcgen05.wait::ld.sync.aligned;")
            for v in range(CH // 8):
                k(f"st.global.v8.b32 [{cptr}+{4 * CH * c + 32 * v}], "
                  f"{{{', '.join(regs[8 * v:8 * v + 8])}}};")
        if HALF:
            k.mark(skip_half)
        # this warp's reads of the buffer are complete: release it to the MMA
        k("tcgen05.fence::before_thread_sync;")
        k("bar.warp.sync 0xffffffff;")
        eae = k.reg("r")
        k(f"mad.lo.u32 {eae}, {ebuf}, 8, {lead_ae};")
        k(f"@{pl0} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{eae}];")

    def emit_tf32_atm_converters():
        """3xTF32 with A in tensor memory.  Warps 4-7: per stage, thread r
        (row r of this CTA's A rows, its TMEM lane) reads the row's BK raw
        values from the swizzled stage and stores them and their low parts
        into the stage's TMEM columns; before converting tile i they drain
        tile i-1 (one accumulator: tile i's MMAs wait for it).  Warps 2-3:
        the low parts of this CTA's B half, into shared memory as before.
        Every converter warp arrives once a stage on the leader's conv
        barrier."""
        lead_conv = k.reg("r")                    # conv[0] of the leader
        k(f"add.u32 {lead_conv}, {bars}, {16 * S};")
        k(f"mapa.shared::cluster.u32 {lead_conv}, {lead_conv}, 0;")
        ntp1 = k.reg("r")
        k(f"add.u32 {ntp1}, {ntile}, 1;")
        b_part = k.label("B_CONV")
        k(f"@!{pepi} bra {b_part};")
        # ---- warps 4-7: A rows into TMEM, drains
        r_ = k.reg("r")
        k(f"mad.lo.u32 {r_}, {q}, 32, {lane};")   # this thread's A row (its TMEM lane)
        rsw = k.reg("r")
        k(f"and.b32 {rsw}, {r_}, 7;")
        roff = k.reg("r")
        k(f"shl.b32 {roff}, {r_}, 7;")            # 128 bytes a row
        ctl = k.reg("r")                          # this warp's TMEM lanes, A columns
        k(f"shl.b32 {ctl}, {q}, 21;")
        k(f"add.u32 {ctl}, {ctl}, {tmem};")
        k(f"add.u32 {ctl}, {ctl}, {ABASE};")
        chunk = []                                # byte offset of K chunk c in the row
        for c in range(BK * 4 // 16):
            # fresh registers (no in-place update), so the static race
            # checker resolves the converters' shared-memory addresses
            x, sh, o = k.reg("r"), k.reg("r"), k.reg("r")
            k(f"xor.b32 {x}, {rsw}, {c};")
            k(f"shl.b32 {sh}, {x}, 4;")
            k(f"add.u32 {o}, {sh}, {roff};")
            chunk.append(o)
        k(f"mov.u32 {st}, 0;")
        k(f"mov.u32 {ph}, 0;")
        atop = tile_loop_head("ATILE")
        pd = k.reg("p")
        k(f"setp.ne.u32 {pd}, {it}, 0;")
        no_drain = k.label("A_NO_DRAIN")
        k(f"@!{pd} bra {no_drain};")
        prev = k.reg("r")
        k(f"sub.u32 {prev}, {it}, 1;")
        epilogue(prev)
        k.mark(no_drain)
        pc = k.reg("p")
        k(f"setp.lt.u32 {pc}, {it}, {ntile};")
        a_skip = k.label("A_SKIP")
        k(f"@!{pc} bra {a_skip};")
        k(f"mov.u32 {kt}, 0;")
        ak = k.label("AK")
        k.mark(ak)
        GemmTemplate._wait(k, bar_addr(0, st), ph, status, 4, teardown)
        # the stage's TMEM columns were last read by MMAs that completed
        # before this stage's copies were issued
        k("tcgen05.fence::after_thread_sync;")
        sba = stage_base(st)
        hi = []
        for c in range(BK * 4 // 16):
            x = k.regs("r", 4)
            ad = k.reg("r")
            k(f"add.u32 {ad}, {sba}, {chunk[c]};")
            k(f"ld.shared.v4.b32 {{{', '.join(x)}}}, [{ad}];")
            hi += x
        lo = []
        for c in range(0, BK, 4):
            lo += tf32_lo_trunc(k, hi[c:c + 4])
        tcol = k.reg("r")
        k(f"mad.lo.u32 {tcol}, {st}, {2 * BK}, {ctl};")
        k(f"tcgen05.st.sync.aligned.32x32b.x{BK}.b32 [{tcol}], {{{', '.join(hi)}}};")
        k(f"tcgen05.st.sync.aligned.32x32b.x{BK}.b32 [{tcol}+{BK}], {{{', '.join(lo)}}};")
        k("tcgen05.wait::st.sync.aligned;")
        k("tcgen05.fence::before_thread_sync;")
        k("bar.warp.sync 0xffffffff;")
        cv = k.reg("r")
        k(f"mad.lo.u32 {cv}, {st}, 8, {lead_conv};")
        k(f"@{pl0} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{cv}];")
        k_loop_tail(ak)
        k.mark(a_skip)
        tile_loop_tail(atop, ntp1)
        k(f"bra {teardown};")
        # ---- warps 2-3: low parts of this CTA's B half into shared memory
        k.mark(b_part)
        CTB = 64
        btid = k.reg("r")
        k(f"sub.u32 {btid}, {tid}, 64;")          # warps 2-3: threads 0..63
        boff = k.reg("r")
        k(f"shl.b32 {boff}, {btid}, 4;")
        NVB = SBH // 16
        assert NVB % CTB == 0
        k(f"mov.u32 {st}, 0;")
        k(f"mov.u32 {ph}, 0;")
        btop = tile_loop_head("BTILE")
        k(f"mov.u32 {kt}, 0;")
        bk = k.label("BK")
        k.mark(bk)
        GemmTemplate._wait(k, bar_addr(0, st), ph, status, 4, teardown)
        sbb = stage_base(st)
        b1, b0 = k.reg("r"), k.reg("r")
        k(f"add.u32 {b1}, {sbb}, {SA};")
        k(f"add.u32 {b0}, {b1}, {boff};")
        for i in range(NVB // CTB):
            x = k.regs("r", 4)
            ad = f"{b0}+{i * 16 * CTB}" if i else b0
            k(f"ld.shared.v4.b32 {{{', '.join(x)}}}, [{ad}];")
            lo = tf32_lo_trunc(k, x)
            k(f"st.shared.v4.b32 [{b0}+{RAW + i * 16 * CTB}], {{{', '.join(lo)}}};")
        k("fence.proxy.async.shared::cta;")
        k("bar.warp.sync 0xffffffff;")
        cvb = k.reg("r")
        k(f"mad.lo.u32 {cvb}, {st}, 8, {lead_conv};")
        k(f"@{pl0} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{cvb}];")
        k_loop_tail(bk)
        tile_loop_tail(btop)

    if not tf32:
        etop = tile_loop_head("ETILE")
        epilogue(it)
        tile_loop_tail(etop)
    elif ATM:
        emit_tf32_atm_converters()
    else:
        # iteration i converts tile i's k-slices (i < ntile), then drains tile
        # i-1 (i >= 1): the drain overlaps the MMAs of tile i's last stages
        lead_conv = k.reg("r")                    # conv[0] of the leader
        k(f"add.u32 {lead_conv}, {bars}, {16 * S};")
        k(f"mapa.shared::cluster.u32 {lead_conv}, {lead_conv}, 0;")
        CT = 32 * CONVW                           # converter threads
        ct = k.reg("r")
        k(f"sub.u32 {ct}, {tid}, {256 - CT};")    # converter thread 0..CT-1
        off0 = k.reg("r")
        k(f"shl.b32 {off0}, {ct}, 4;")            # 16 bytes per thread per pass
        NV = RAW // 16                            # 16-byte vectors per stage
        ptail = k.reg("p")                        # threads of the partial last pass
        k(f"setp.lt.u32 {ptail}, {ct}, {NV % CT};")
        ntp1 = k.reg("r")
        k(f"add.u32 {ntp1}, {ntile}, 1;")
        k(f"mov.u32 {st}, 0;")
        k(f"mov.u32 {ph}, 0;")
        ctop = tile_loop_head("CTILE")
        pconv = k.reg("p")
        k(f"setp.lt.u32 {pconv}, {it}, {ntile};")
        skip_conv = k.label("SKIP_CONV")
        k(f"@!{pconv} bra {skip_conv};")
        k(f"mov.u32 {kt}, 0;")
        ck = k.label("CK")
        k.mark(ck)
        GemmTemplate._wait(k, bar_addr(0, st), ph, status, 4, teardown)
        sbc = stage_base(st)
        a0 = k.reg("r")
        k(f"add.u32 {a0}, {sbc}, {off0};")
        def convert(i):
            x = k.regs("r", 4)
            ad = f"{a0}+{i * 16 * CT}" if i else a0
            k(f"ld.shared.v4.b32 {{{', '.join(x)}}}, [{ad}];")
            if _gemm.TF32_HI_RAW:
                lo = tf32_lo_trunc(k, x)
            else:
                hi, lo = tf32_split(k, x)
                k(f"st.shared.v4.b32 [{ad}], {{{', '.join(hi)}}};")
            k(f"st.shared.v4.b32 [{a0}+{RAW + i * 16 * CT}], {{{', '.join(lo)}}};")
        for i in range(NV // CT):
            convert(i)
        if NV % CT:
            skip_tail = k.label("CONV_TAIL")
            k(f"@!{ptail} bra {skip_tail};")
            convert(NV // CT)
            k.mark(skip_tail)
        # generic-proxy stores -> the tensor core's async-proxy reads
        k("fence.proxy.async.shared::cta;")
        k("bar.warp.sync 0xffffffff;")
        cv = k.reg("r")
        k(f"mad.lo.u32 {cv}, {st}, 8, {lead_conv};")
        k(f"@{pl0} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{cv}];")
        k_loop_tail(ck)
        k.mark(skip_conv)
        pdrain = k.reg("p")
        k(f"setp.ne.u32 {pdrain}, {it}, 0;")
        k(f"and.pred {pdrain}, {pdrain}, {pepi};")    # the drain: warps 4-7
        skip_drain = k.label("SKIP_DRAIN")
        k(f"@!{pdrain} bra {skip_drain};")
        prev = k.reg("r")
        k(f"sub.u32 {prev}, {it}, 1;")
        epilogue(prev)
        k.mark(skip_drain)
        tile_loop_tail(ctop, ntp1)

    # ---------------- teardown ----------------
    k.mark(teardown)
    k("tcgen05.fence::before_thread_sync;")
    k("barrier.sync 0;")
    k("barrier.cluster.arrive.release;")
    k("barrier.cluster.wait.acquire;")
    end = k.label("END")
    k(f"@!{pw1} bra {end};")
    k("bar.warp.sync 0xffffffff;")
    k("tcgen05.fence::after_thread_sync;")
    k(f"tcgen05.dealloc.cta_group::2.sync.aligned.b32 {tmem}, 512;")
    k.mark(end)
    k.mark(idle)
    k("ret;")
    return k.render()

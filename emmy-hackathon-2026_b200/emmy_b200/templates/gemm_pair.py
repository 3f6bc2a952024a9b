"""bf16 matmul on CTA pairs: ``tcgen05.mma.cta_group::2``, 256 x 256 per pair.

The IR's schedule gives every CTA a 128 x 256 output tile (reference
``problems/m01_matmul_512/*.ir.txt:1-37`` form).  Two such CTAs whose tiles
are vertical neighbours (rows ``256*p .. 256*p+255`` of the same 256 columns)
form a cluster of 2 and compute their 256 x 256 block as ONE pair MMA:

* each CTA loads, per k-slice, its own 128 rows of A (16 KiB) and HALF of the
  pair's B slice (64 k-rows x 128 columns, 16 KiB) into the same offset of its
  own shared memory, so a stage is 32 KiB instead of the 48 KiB a lone CTA
  needs for 128 x 256 -- B is read from L2/HBM once per pair, not twice;
* the TMA copies of both CTAs (``.cta_group::2`` form, each into its own CTA) count
  their bytes on the LEADER's ``full`` mbarrier (address from ``mapa``); only
  the leader arms it (``expect_tx`` of both CTAs' bytes);
* one thread of the leader issues ``tcgen05.mma.cta_group::2.kind::f16``
  (M=256, N=256, K=16): A rows come from both CTAs' shared memory, B columns
  from both halves, and each CTA's tensor memory receives its 128 rows x 256
  columns of f32 accumulators (allocated by ``tcgen05.alloc.cta_group::2``
  in both CTAs);
* ``tcgen05.commit`` in its cluster-multicast form, CTA mask 0b11, releases a
  stage in BOTH CTAs' ``empty`` barriers, and at the end signals both CTAs'
  ``acc`` barriers; each CTA then drains its own tensor memory exactly like
  the single-CTA template (``tcgen05.ld.32x32b.x32``, ``st.global.v8``).

Pair p (CTAs 2p and 2p+1) takes pair tile p in the grouped order of
``gemm_persistent.raster``.  Cluster barriers (``barrier.cluster``) order the mbarrier initialisation and
tensor-memory allocation before any cross-CTA traffic, and keep each CTA
alive until its peer is done with it.  Every mbarrier wait is bounded by
``%globaltimer`` as in the single-CTA template (codes 1 producer, 2 MMA
issuer, 3 epilogue, 5 MMA drain).
"""
from __future__ import annotations

from ..ptx import Kernel
from .gemm import GemmTemplate, _desc_hi, idesc_mma

PAIR_STAGE_MAX = 6
PAIR_STAGE = 128 * 64 * 2 + 64 * 128 * 2      # A slice + B half, bf16: 32 KiB


def pair_stages(smem_bytes: int, limit: int, stage: int = PAIR_STAGE) -> int:
    """Ring depth the meta's dynamic shared memory allows (1 KiB alignment
    slack and 256 B of barriers are set aside); ``stage`` is one CTA's bytes
    per stage (3xTF32: 64 KiB, raw slices plus their low parts)."""
    return min(PAIR_STAGE_MAX, (min(smem_bytes, limit) - 1024 - 256) // stage)


def emit_pair(t) -> str:
    ctx = t.ctx
    BM, BN, BK, S, K = 128, 256, 64, t.pair_S, t.K
    KT = K // BK
    SA = BM * BK * 2                 # own A rows: 16 KiB
    SBH = BK * 128 * 2               # own half of B: 64 k-rows x 128 columns
    STG = SA + SBH
    BOXN = 64                        # B boxes are 128 bytes (64 bf16) wide
    params = ctx.params() + [("tmapA", ".align 64 .b8", "[128]"),
                             ("tmapB", ".align 64 .b8", "[128]")]
    k = Kernel(ctx.entry, params)
    k.maxntid = (256, 1, 1)
    k.reqnctapercluster = (2, 1, 1)
    k.directive("cluster 2 1 1")
    k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
    k.decl(".global .align 4 .u32 __emmy_status;")
    k.directive(f"tmap tmapA buf={t.A} dtype=9 dims={K},{t.M} strides={K * 2} "
                f"box={BK},{BM} swizzle=3")
    k.directive(f"tmap tmapB buf={t.B} dtype=9 dims={t.N},{K} strides={t.N * 2} "
                f"box={BOXN},{BK} swizzle=3")
    k.comment(f"emmy-b200 template: tcgen05 gemm bf16 M={t.M} N={t.N} K={K} on CTA pairs, "
              f"256x256x{BK} per pair, stages={S}")
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
    cta = k.special("%ctaid.x")
    pair = k.reg("r")
    k(f"shr.u32 {pair}, {cta}, 1;")
    from .gemm_persistent import raster
    mp, nbk = raster(k, pair, t.M // 256, t.NB)
    m0 = k.reg("r")                              # (2 * mp + rank) * 128
    k(f"mad.lo.u32 {m0}, {mp}, 2, {rank};")
    k(f"mul.lo.u32 {m0}, {m0}, {BM};")
    n0 = k.reg("r")
    k(f"mul.lo.u32 {n0}, {nbk}, {BN};")
    nh = k.reg("r")                              # this CTA's half of the B columns
    k(f"mad.lo.u32 {nh}, {rank}, 128, {n0};")
    plead = k.reg("p")
    k(f"setp.eq.u32 {plead}, {rank}, 0;")
    # shared memory: S stages of [A 16K | B half 16K], then the mbarriers
    # full[S], empty[S], acc, drain and the tensor-memory slot
    raw = k.reg("r")
    k(f"mov.u32 {raw}, __emmy_smem;")
    ring = k.reg("r")
    k(f"add.u32 {ring}, {raw}, 1023;")
    k(f"and.b32 {ring}, {ring}, -1024;")
    bars = k.reg("r")
    k(f"add.u32 {bars}, {ring}, {S * STG};")
    accb = k.reg("r")
    k(f"add.u32 {accb}, {bars}, {16 * S};")
    drain = k.reg("r")
    k(f"add.u32 {drain}, {accb}, 8;")
    tslot = k.reg("r")
    k(f"add.u32 {tslot}, {accb}, 16;")
    status = k.reg("rd")
    k(f"mov.u64 {status}, __emmy_status;")
    p0 = k.reg("p")
    k(f"setp.eq.u32 {p0}, {tid}, 0;")
    skip_init = k.label("SKIP_INIT")
    k(f"@!{p0} bra {skip_init};")
    for s in range(2 * S):
        k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], 1;")
    k(f"mbarrier.init.shared::cta.b64 [{accb}], 1;")
    k(f"mbarrier.init.shared::cta.b64 [{drain}], 1;")
    k("fence.mbarrier_init.release.cluster;")
    k(f"prefetch.tensormap [{ta}];")
    k(f"prefetch.tensormap [{tb}];")
    k.mark(skip_init)
    pw1 = k.reg("p")
    k(f"setp.eq.u32 {pw1}, {warp}, 1;")
    skip_alloc = k.label("SKIP_ALLOC")
    k(f"@!{pw1} bra {skip_alloc};")
    # warp 1 of both CTAs allocates collectively: the same 256 columns in each
    k(f"tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [{tslot}], 256;")
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
    kt, st, ph = k.reg("r"), k.reg("r"), k.reg("r")

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

    def loop_head(label):
        k(f"mov.u32 {kt}, 0;")
        k(f"mov.u32 {st}, 0;")
        k(f"mov.u32 {ph}, 0;")
        top = k.label(label)
        k.mark(top)
        return top

    def loop_tail(top):
        GemmTemplate._advance(k, st, ph, S)
        k(f"add.u32 {kt}, {kt}, 1;")
        pl = k.reg("p")
        k(f"setp.lt.u32 {pl}, {kt}, {KT};")
        k(f"@{pl} bra {top};")

    # ---------------- producer: warp 0, lane 0 of both CTAs ----------------
    pprod = k.reg("p")
    k(f"setp.eq.u32 {pprod}, {warp}, 0;")
    k(f"and.pred {pprod}, {pprod}, {pl0};")
    end_prod = k.label("END_PROD")
    k(f"@!{pprod} bra {end_prod};")
    lead_full = k.reg("r")                       # full[0] of the leader CTA
    k(f"mapa.shared::cluster.u32 {lead_full}, {bars}, 0;")
    top = loop_head("PROD")
    par = k.reg("r")
    k(f"xor.b32 {par}, {ph}, 1;")
    GemmTemplate._wait(k, bar_addr(1, st), par, status, 1, end_prod)
    fb = k.reg("r")
    k(f"mad.lo.u32 {fb}, {st}, 8, {lead_full};")
    own_fb = bar_addr(0, st)
    k(f"@{plead} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{own_fb}], {2 * STG};")
    kc = k.reg("r")
    k(f"mul.lo.u32 {kc}, {kt}, {BK};")
    da = stage_base(st)
    k(f"cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      f"[{da}], [{ta}, {{{kc}, {m0}}}], [{fb}];")
    for i in range(2):
        nx = k.reg("r")
        k(f"add.u32 {nx}, {nh}, {BOXN * i};")
        db = k.reg("r")
        k(f"add.u32 {db}, {da}, {SA + i * BK * 128};")
        k(f"cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx"
          f"::bytes [{db}], [{tb}, {{{nx}, {kc}}}], [{fb}];")
    loop_tail(top)
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
    idesc = k.reg("r")
    k(f"mov.u32 {idesc}, {idesc_mma(2 * BM, BN, True)};")
    hiA = _desc_hi(16, 1024)
    hiB = _desc_hi(BK * 128, 1024)
    top2 = loop_head("MMA")
    GemmTemplate._wait(k, bar_addr(0, st), ph, status, 2, end_mma)
    k("tcgen05.fence::after_thread_sync;")
    sb = stage_base(st)
    bad = k.reg("r")
    k(f"add.u32 {bad}, {sb}, {SA};")
    adesc = GemmTemplate._desc(k, sb, hiA)
    bdesc = GemmTemplate._desc(k, bad, hiB)
    pacc = k.reg("p")
    k(f"setp.ne.u32 {pacc}, {kt}, 0;")
    ptrue = k.reg("p")
    k(f"setp.eq.u32 {ptrue}, 0, 0;")
    for kk in range(BK // 16):
        ad = k.reg("rd")
        k(f"add.s64 {ad}, {adesc}, {kk * 2};")          # +32 B along K
        bd = k.reg("rd")
        k(f"add.s64 {bd}, {bdesc}, {kk * 16 * 8};")     # +16 k-rows of 128 B
        k(f"tcgen05.mma.cta_group::2.kind::f16 [{tmem}], {ad}, {bd}, {idesc}, "
          f"{pacc if kk == 0 else ptrue};")
    k(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      f"[{bar_addr(1, st)}], {mask};")
    loop_tail(top2)
    k(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      f"[{accb}], {mask};")
    # the issuing thread also waits for its own MMAs to finish before it leaves
    k(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [{drain}];")
    zero_d = k.reg("r")
    k(f"mov.u32 {zero_d}, 0;")
    GemmTemplate._wait(k, drain, zero_d, status, 5, end_mma)
    k.mark(end_mma)

    # ---------------- epilogue: all 8 warps of each CTA ----------------
    k("bar.warp.sync 0xffffffff;")
    zero = k.reg("r")
    k(f"mov.u32 {zero}, 0;")
    GemmTemplate._wait(k, accb, zero, status, 3, teardown)
    k("tcgen05.fence::after_thread_sync;")
    q = k.reg("r")
    k(f"and.b32 {q}, {warp}, 3;")
    h = k.reg("r")
    k(f"shr.u32 {h}, {warp}, 2;")
    row = k.reg("r")
    k(f"mad.lo.u32 {row}, {q}, 32, {lane};")
    k(f"add.u32 {row}, {row}, {m0};")
    half = BN // 2
    col = k.reg("r")
    k(f"mad.lo.u32 {col}, {h}, {half}, {n0};")
    taddr = k.reg("r")
    k(f"shl.b32 {taddr}, {q}, 21;")              # (32*q) << 16: TMEM lane field
    hc = k.reg("r")
    k(f"mul.lo.u32 {hc}, {h}, {half};")
    k(f"add.u32 {taddr}, {taddr}, {hc};")
    k(f"add.u32 {taddr}, {taddr}, {tmem};")
    off = k.reg("rd")
    k(f"mul.wide.u32 {off}, {row}, {t.N * 4};")
    c2 = k.reg("rd")
    k(f"mul.wide.u32 {c2}, {col}, 4;")
    k(f"add.s64 {off}, {off}, {c2};")
    cptr = k.reg("rd")
    k(f"add.s64 {cptr}, {cbase}, {off};")
    for c in range(half // 32):
        regs = k.regs("r", 32)
        ta2 = k.reg("r")
        k(f"add.u32 {ta2}, {taddr}, {32 * c};")
        k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{ta2}];")
        k("tcgen05.wait::ld.sync.aligned;")
        for v in range(4):
            k(f"st.global.v8.b32 [{cptr}+{128 * c + 32 * v}], "
              f"{{{', '.join(regs[8 * v:8 * v + 8])}}};")
    # ---------------- teardown ----------------
    # possibly diverged after a timed-out wait: non-aligned barriers; the
    # cluster barrier keeps this CTA's shared and tensor memory alive until
    # the peer is done with them
    k.mark(teardown)
    k("tcgen05.fence::before_thread_sync;")
    k("barrier.sync 0;")
    k("barrier.cluster.arrive.release;")
    k("barrier.cluster.wait.acquire;")
    end = k.label("END")
    k(f"@!{pw1} bra {end};")
    k("bar.warp.sync 0xffffffff;")
    k("tcgen05.fence::after_thread_sync;")
    k(f"tcgen05.dealloc.cta_group::2.sync.aligned.b32 {tmem}, 256;")
    k.mark(end)
    k("ret;")
    return k.render()

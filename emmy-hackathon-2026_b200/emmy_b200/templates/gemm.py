"""Matmul template: ``C = A @ B`` on the 5th-generation tensor cores.

Matches Emmy's shared-memory matmul schedule (reference
``problems/m01_matmul_512/*.ir.txt:1-37``: a CTA per BM x BN output tile,
``Init`` accumulators, ``CpAsyncCopy`` of A/B k-slices into ``Smem``, an inner
``Loop`` of ``multiply`` + ``Accum add`` over shared-memory loads, then the
micro-tile ``Write``s).  The reference lowers that IR to CUDA-core FFMAs with
a cp.async ring (``stmt_cpasync_copy`` ``compile.py:1754-1772``, full unroll
``:1882-1928``, FMA contraction ``:2250-2264``).  This template keeps the
IR's CTA -> output-tile assignment and computes each tile with:

* TMA (``cp.async.bulk.tensor.2d``, no multicast) loading 128-byte-swizzled
  A and B k-slices into an S-stage shared-memory ring, one elected thread,
  completion counted on an mbarrier (``complete_tx``);
* one elected thread issuing ``tcgen05.mma.cta_group::1.kind::f16`` (bf16
  inputs, f32 accumulate; M=128, N=BN, K=16 per instruction) with the
  accumulator in tensor memory (``tcgen05.alloc``), each stage released back
  to the producer by ``tcgen05.commit`` on its ``empty`` mbarrier;
* all warps draining TMEM with ``tcgen05.ld.32x32b.x32`` (warp w reads lanes
  32*(w%4)..+31, i.e. output rows) and writing 32-byte ``st.global.v8`` rows.

A is K-major ([M,K] row-major) and B MN-major ([K,N] row-major), both with
the 128-byte swizzle; the shared-memory matrix descriptors follow the UMMA
canonical layouts (K-major: 8-row groups 1024 B apart; MN-major: 64-element
N blocks ``BK*128`` B apart, 8-row K groups 1024 B apart).

Every mbarrier wait is bounded by ``%globaltimer`` (2 s); on expiry the
kernel records a code in the module-scope word ``__emmy_status`` (1 producer,
2 MMA issuer, 3 epilogue) and the thread leaves its role: the producer and
MMA threads rejoin their warps at the end of their role, the epilogue goes
to the teardown, which frees TMEM, so a stalled pipeline returns an error
instead of hanging the GPU.  Tensor maps are built on the host
(``// @emmy tmap`` directives; reference ``TASK.md:130`` declares
``TmaDescriptor`` host-built) and passed after the meta ``arg_order``
parameters.
"""
from __future__ import annotations

from ..analysis import NotAffine, affine, kind, walk
from ..ir import dim
from ..ptx import Kernel
from .common import TemplateMismatch

WAIT_NS = 2_000_000_000       # bounded mbarrier waits: 2 s of %globaltimer
SMEM_LIMIT = 227 * 1024       # max dynamic shared memory per CTA on sm_100


def _desc_hi(lbo: int, sbo: int, swizzle_code: int = 2) -> int:
    """Constant part of a UMMA shared-memory descriptor: leading/stride byte
    offsets (>>4), descriptor version 1 (bits 46-47), layout type at 61-63
    (2 = 128-byte swizzle); the start address (>>4) is added at run time."""
    return ((lbo >> 4) << 16) | ((sbo >> 4) << 32) | (1 << 46) | (swizzle_code << 61)


def idesc_f16(M: int, N: int, b_mn_major: bool) -> int:
    """Instruction descriptor of ``tcgen05.mma .kind::f16``: f32 accumulator
    (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), A K-major, B major-ness
    at bit 16, N>>3 at bits 17-22, M>>4 at bits 24-28."""
    return (1 << 4) | (1 << 7) | (1 << 10) | (int(b_mn_major) << 16) | ((N >> 3) << 17) \
        | ((M >> 4) << 24)


class GemmTemplate:
    name = "gemm"

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "GemmTemplate":
        tile = ctx.tile
        if tile is None:
            raise TemplateMismatch("no single top-level Tile")
        axes = ctx.tile_axes()
        names = [a for a, _ in axes]
        if names != ["a0_b", "a1_b", "a0_u", "a1_u"]:
            raise TemplateMismatch("not a matmul tile (a0_b, a1_b, a0_u, a1_u)")
        ext = dict(axes)
        body = list(walk(tile.body))
        inits = [s for s in body if kind(s) == "Init"]
        copies = [s for s in body if kind(s) == "CpAsyncCopy"]
        smems = {s.name for s in body if kind(s) == "Smem"}
        writes = [s for s in body if kind(s) == "Write"]
        if not inits or not copies or len(smems) != 2 or not writes:
            raise TemplateMismatch("matmul statements missing")
        bufs = ctx.bufs
        src_of = {}
        for c in copies:
            if c.smem not in smems:
                raise TemplateMismatch("copy into undeclared smem")
            if src_of.setdefault(c.smem, c.src) != c.src:
                raise TemplateMismatch("smem filled from two buffers")
        accs = {s.name for s in inits}
        if any(float(s.identity) != 0.0 for s in inits):
            raise TemplateMismatch("accumulator not zero-initialised")
        # the contraction: acc += multiply(load smemX, load smemY)
        loops = [s for s in body if kind(s) == "Loop"]
        if len(loops) != 1:
            raise TemplateMismatch("expected one inner k loop")
        defs = {}
        pairs = set()
        role = {}          # smem tile -> "A" (indexed by a0_u) / "B" (by a1_u)
        for s in loops[0].body:
            k = kind(s)
            if k == "Load":
                if s.input not in smems:
                    raise TemplateMismatch("inner loop reads global memory")
                defs[s.names[0]] = ("load", s.input)
                fv = set()
                for ix in s.index:
                    fv |= ix.free_vars() if hasattr(ix, "free_vars") else set()
                r = "A" if "a0_u" in fv and "a1_u" not in fv else \
                    "B" if "a1_u" in fv and "a0_u" not in fv else None
                if r is None or role.setdefault(s.input, r) != r:
                    raise TemplateMismatch("operand tile indexing")
            elif k == "Assign":
                if s.op.name != "multiply" or len(s.args) != 2:
                    raise TemplateMismatch(f"inner op {s.op.name}")
                a, b = (defs.get(x) for x in s.args)
                if not (a and b and a[0] == b[0] == "load" and a[1] != b[1]):
                    raise TemplateMismatch("multiply of non-smem operands")
                defs[s.name] = ("mul", frozenset((a[1], b[1])))
            elif k == "Accum":
                if s.name not in accs or s.op.name != "add" or s.base:
                    raise TemplateMismatch("accumulate shape")
                v = defs.get(s.value)
                if not v or v[0] != "mul":
                    raise TemplateMismatch("accumulate of a non-product")
                pairs.add(v[1])
            else:
                raise TemplateMismatch(f"{k} in the inner k loop")
        if pairs != {frozenset(smems)}:
            raise TemplateMismatch("products do not pair the two smem tiles")
        outs = {w.output for w in writes}
        if len(outs) != 1 or any(w.atomic for w in writes):
            raise TemplateMismatch("split-k / multiple outputs")
        C = outs.pop()
        if bufs.dtypes.get(C) != "f32" or len(bufs.shapes[C]) != 2:
            raise TemplateMismatch("output")
        M, N = bufs.shapes[C]
        inv = {v: s for s, v in role.items()}
        if set(inv) != {"A", "B"}:
            raise TemplateMismatch("operand roles")
        A, B = src_of.get(inv["A"]), src_of.get(inv["B"])
        if A is None or B is None or len(bufs.shapes[A]) != 2 or len(bufs.shapes[B]) != 2 or \
                bufs.shapes[A][0] != M or bufs.shapes[B][1] != N or \
                bufs.shapes[A][1] != bufs.shapes[B][0]:
            raise TemplateMismatch("operand shapes")
        K = bufs.shapes[A][1]
        # output tile of a CTA from the write indices
        BM = BN = None
        for w in writes:
            try:
                r = affine(w.index[0])
                c = affine(w.index[1])
            except NotAffine as e:
                raise TemplateMismatch(str(e))
            if BM is None:
                BM, BN = r.coef("a0_b"), c.coef("a1_b")
            if r.coef("a0_b") != BM or c.coef("a1_b") != BN:
                raise TemplateMismatch("write tile")
        if (BM, BN) == (None, None) or ext["a0_b"] * BM != M or ext["a1_b"] * BN != N:
            raise TemplateMismatch("tile does not cover the output")
        dts = {bufs.dtypes[A], bufs.dtypes[B]}
        if dts != {"bf16"}:
            raise TemplateMismatch(f"operand dtype {dts} (bf16 path)")
        threads = ctx.threads
        if ctx.block != (threads, 1, 1) or threads != 256:
            raise TemplateMismatch("tcgen05 template runs 256-thread CTAs")
        if ctx.grid[0] * ctx.grid[1] * ctx.grid[2] != ext["a0_b"] * ext["a1_b"]:
            raise TemplateMismatch("grid is not one CTA per output tile")
        if BM != 128 or BN % 64 or not 64 <= BN <= 256 or K % 64:
            raise TemplateMismatch(f"tile {BM}x{BN}, K={K} outside the tcgen05 shapes")
        self = cls()
        self.ctx, self.A, self.B, self.C = ctx, A, B, C
        self.M, self.N, self.K, self.BM, self.BN = M, N, K, BM, BN
        self.BK = 64
        self.esize = 2
        stage = (BM * self.BK + self.BK * BN) * self.esize
        self.stage_bytes = stage
        avail = min(ctx.smem_bytes, SMEM_LIMIT) - 1024 - 256
        self.S = min(6, avail // stage)
        if self.S < 2:
            raise TemplateMismatch("meta smem_bytes too small for a 2-stage ring")
        self.NB = ext["a1_b"]
        return self

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        ctx = self.ctx
        BM, BN, BK, S, K = self.BM, self.BN, self.BK, self.S, self.K
        KT = K // BK
        SA = BM * BK * 2                 # A stage bytes (16 KB)
        SB = BK * BN * 2                 # B stage bytes
        NBOX = BN // 64                  # B loaded as 64-column boxes
        params = ctx.params() + [("tmapA", ".align 64 .b8", "[128]"),
                                 ("tmapB", ".align 64 .b8", "[128]")]
        k = Kernel(ctx.entry, params)
        k.maxntid = (256, 1, 1)
        k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
        k.decl(".global .align 4 .u32 __emmy_status;")
        # host-built tensor maps (innermost dimension first)
        k.directive(f"tmap tmapA buf={self.A} dtype=9 dims={K},{self.M} strides={K * 2} "
                    f"box={BK},{BM} swizzle=3")
        k.directive(f"tmap tmapB buf={self.B} dtype=9 dims={self.N},{K} strides={self.N * 2} "
                    f"box=64,{BK} swizzle=3")
        k.comment(f"emmy-b200 template: tcgen05 gemm bf16 M={self.M} N={self.N} K={K} "
                  f"tile {BM}x{BN}x{BK} stages={S}")
        cbase = k.param_ptr(self.C)
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
        cta = k.special("%ctaid.x")
        mblk = k.reg("r")
        k(f"div.u32 {mblk}, {cta}, {self.NB};")
        nblk = k.reg("r")
        k(f"rem.u32 {nblk}, {cta}, {self.NB};")
        m0 = k.reg("r")
        k(f"mul.lo.u32 {m0}, {mblk}, {BM};")
        n0 = k.reg("r")
        k(f"mul.lo.u32 {n0}, {nblk}, {BN};")
        # shared memory layout (1024-aligned base): A ring, B ring, barriers
        raw = k.reg("r")
        k(f"mov.u32 {raw}, __emmy_smem;")
        base = k.reg("r")
        k(f"add.u32 {base}, {raw}, 1023;")
        k(f"and.b32 {base}, {base}, -1024;")
        a_ring = base
        b_ring = k.reg("r")
        k(f"add.u32 {b_ring}, {base}, {S * SA};")
        bars = k.reg("r")
        k(f"add.u32 {bars}, {b_ring}, {S * SB};")
        # full[s] at bars + 8s, empty[s] at bars + 8(S+s), accum at bars + 16S,
        # tmem address slot at bars + 16S + 8
        accb = k.reg("r")
        k(f"add.u32 {accb}, {bars}, {16 * S};")
        tslot = k.reg("r")
        k(f"add.u32 {tslot}, {bars}, {16 * S + 8};")
        status = k.reg("rd")
        k(f"mov.u64 {status}, __emmy_status;")
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip_init = k.label("SKIP_INIT")
        k(f"@!{p0} bra {skip_init};")
        for s in range(2 * S + 1):
            k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], 1;")
        k("fence.mbarrier_init.release.cluster;")
        k(f"prefetch.tensormap [{ta}];")
        k(f"prefetch.tensormap [{tb}];")
        k.mark(skip_init)
        pw1 = k.reg("p")
        k(f"setp.eq.u32 {pw1}, {warp}, 1;")
        skip_alloc = k.label("SKIP_ALLOC")
        k(f"@!{pw1} bra {skip_alloc};")
        k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{tslot}], {max(32, BN)};")
        k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
        k.mark(skip_alloc)
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
        k("tcgen05.fence::after_thread_sync;")
        tmem = k.reg("r")
        k(f"ld.shared.u32 {tmem}, [{tslot}];")
        teardown = k.label("TEARDOWN")

        # ---------------- producer: warp 0, lane 0 ----------------
        pl0 = k.reg("p")
        k(f"setp.eq.u32 {pl0}, {lane}, 0;")
        pprod = k.reg("p")
        k(f"setp.eq.u32 {pprod}, {warp}, 0;")
        k(f"and.pred {pprod}, {pprod}, {pl0};")
        end_prod = k.label("END_PROD")
        k(f"@!{pprod} bra {end_prod};")
        kt = k.reg("r")
        st = k.reg("r")
        ph = k.reg("r")
        k(f"mov.u32 {kt}, 0;")
        k(f"mov.u32 {st}, 0;")
        k(f"mov.u32 {ph}, 0;")
        top = k.label("PROD")
        k.mark(top)
        eb = k.reg("r")
        k(f"mad.lo.u32 {eb}, {st}, 8, {bars};")
        k(f"add.u32 {eb}, {eb}, {8 * S};")
        par = k.reg("r")
        k(f"xor.b32 {par}, {ph}, 1;")
        self._wait(k, eb, par, status, 1, end_prod)
        fb = k.reg("r")
        k(f"mad.lo.u32 {fb}, {st}, 8, {bars};")
        k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {SA + SB};")
        kc = k.reg("r")
        k(f"mul.lo.u32 {kc}, {kt}, {BK};")
        da = k.reg("r")
        k(f"mad.lo.u32 {da}, {st}, {SA}, {a_ring};")
        k(f"cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
          f"[{da}], [{ta}, {{{kc}, {m0}}}], [{fb}];")
        dbb = k.reg("r")
        k(f"mad.lo.u32 {dbb}, {st}, {SB}, {b_ring};")
        for i in range(NBOX):
            nx = k.reg("r")
            k(f"add.u32 {nx}, {n0}, {64 * i};")
            db = k.reg("r")
            k(f"add.u32 {db}, {dbb}, {i * BK * 128};")
            k(f"cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
              f"[{db}], [{tb}, {{{nx}, {kc}}}], [{fb}];")
        self._advance(k, st, ph, S)
        k(f"add.u32 {kt}, {kt}, 1;")
        pl = k.reg("p")
        k(f"setp.lt.u32 {pl}, {kt}, {KT};")
        k(f"@{pl} bra {top};")
        k.mark(end_prod)

        # ---------------- MMA issuer: warp 1, lane 0 ----------------
        pmma = k.reg("p")
        k(f"setp.eq.u32 {pmma}, {warp}, 1;")
        k(f"and.pred {pmma}, {pmma}, {pl0};")
        end_mma = k.label("END_MMA")
        k(f"@!{pmma} bra {end_mma};")
        idesc = k.reg("r")
        k(f"mov.u32 {idesc}, {idesc_f16(BM, BN, True)};")
        hiA = _desc_hi(16, 1024)
        hiB = _desc_hi(BK * 128, 1024)
        k(f"mov.u32 {kt}, 0;")
        k(f"mov.u32 {st}, 0;")
        k(f"mov.u32 {ph}, 0;")
        top2 = k.label("MMA")
        k.mark(top2)
        fb2 = k.reg("r")
        k(f"mad.lo.u32 {fb2}, {st}, 8, {bars};")
        self._wait(k, fb2, ph, status, 2, end_mma)
        k("tcgen05.fence::after_thread_sync;")
        aad = k.reg("r")
        k(f"mad.lo.u32 {aad}, {st}, {SA}, {a_ring};")
        bad = k.reg("r")
        k(f"mad.lo.u32 {bad}, {st}, {SB}, {b_ring};")
        adesc = self._desc(k, aad, hiA)
        bdesc = self._desc(k, bad, hiB)
        pacc = k.reg("p")
        k(f"setp.ne.u32 {pacc}, {kt}, 0;")
        for kk in range(BK // 16):
            ad = k.reg("rd")
            k(f"add.s64 {ad}, {adesc}, {kk * 2};")          # +32 bytes along K
            bd = k.reg("rd")
            k(f"add.s64 {bd}, {bdesc}, {kk * 128};")        # +16 rows * 128 bytes
            pa = pacc if kk == 0 else "1"
            if kk == 0:
                k(f"tcgen05.mma.cta_group::1.kind::f16 [{tmem}], {ad}, {bd}, {idesc}, {pa};")
            else:
                pt = k.reg("p")
                k(f"setp.eq.u32 {pt}, 0, 0;")
                k(f"tcgen05.mma.cta_group::1.kind::f16 [{tmem}], {ad}, {bd}, {idesc}, {pt};")
        eb2 = k.reg("r")
        k(f"mad.lo.u32 {eb2}, {st}, 8, {bars};")
        k(f"add.u32 {eb2}, {eb2}, {8 * S};")
        k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{eb2}];")
        self._advance(k, st, ph, S)
        k(f"add.u32 {kt}, {kt}, 1;")
        pl2 = k.reg("p")
        k(f"setp.lt.u32 {pl2}, {kt}, {KT};")
        k(f"@{pl2} bra {top2};")
        k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{accb}];")
        k.mark(end_mma)

        # ---------------- epilogue: all 8 warps ----------------
        k("bar.warp.sync 0xffffffff;")
        zero = k.reg("r")
        k(f"mov.u32 {zero}, 0;")
        self._wait(k, accb, zero, status, 3, teardown)
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
        k(f"shl.b32 {taddr}, {q}, 21;")              # (32*q) << 16
        hc = k.reg("r")
        k(f"mul.lo.u32 {hc}, {h}, {half};")
        k(f"add.u32 {taddr}, {taddr}, {hc};")
        k(f"add.u32 {taddr}, {taddr}, {tmem};")
        off = k.reg("rd")
        k(f"mul.wide.u32 {off}, {row}, {self.N * 4};")
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
        # reached converged, or (after a timed-out wait) diverged: the
        # non-aligned barrier tolerates both; warp 1 re-converges before the
        # warp-wide dealloc
        k.mark(teardown)
        k("tcgen05.fence::before_thread_sync;")
        k("barrier.sync 0;")
        end = k.label("END")
        k(f"@!{pw1} bra {end};")
        k("bar.warp.sync 0xffffffff;")
        k("tcgen05.fence::after_thread_sync;")
        k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {max(32, BN)};")
        k.mark(end)
        k("ret;")
        return k.render()

    @staticmethod
    def _advance(k, st, ph, S):
        """stage = (stage + 1) % S, flipping the phase bit on wrap."""
        p = k.reg("p")
        k(f"add.u32 {st}, {st}, 1;")
        k(f"setp.eq.u32 {p}, {st}, {S};")
        k(f"@{p} mov.u32 {st}, 0;")
        k(f"@{p} xor.b32 {ph}, {ph}, 1;")

    @staticmethod
    def _desc(k, addr, hi) -> str:
        lo = k.reg("r")
        k(f"shr.u32 {lo}, {addr}, 4;")
        d = k.reg("rd")
        k(f"cvt.u64.u32 {d}, {lo};")
        k(f"or.b64 {d}, {d}, {hi};")
        return d

    @staticmethod
    def _wait(k, bar, parity, status, code, fail_label):
        """Spin on ``mbarrier.try_wait.parity`` for at most WAIT_NS of
        %globaltimer; on expiry store ``code`` to ``__emmy_status`` and jump
        to ``fail_label``."""
        t0 = k.reg("rd")
        k(f"mov.u64 {t0}, %globaltimer;")
        top, ok = k.label("WAIT"), k.label("WAIT_OK")
        k.mark(top)
        p = k.reg("p")
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar}], {parity};")
        k(f"@{p} bra {ok};")
        t1 = k.reg("rd")
        k(f"mov.u64 {t1}, %globaltimer;")
        k(f"sub.s64 {t1}, {t1}, {t0};")
        q = k.reg("p")
        k(f"setp.lt.s64 {q}, {t1}, {WAIT_NS};")
        k(f"@{q} bra {top};")
        k(f"st.global.u32 [{status}], {code};")
        k(f"bra {fail_label};")
        k.mark(ok)

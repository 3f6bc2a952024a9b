"""Matmul template: ``C = A @ B`` on the 5th-generation tensor cores.

Matches Emmy's shared-memory matmul schedule (reference
``problems/m01_matmul_512/*.ir.txt:1-37``: a CTA per BM x BN output tile,
``Init`` accumulators, ``CpAsyncCopy`` of A/B k-slices into ``Smem``, an inner
``Loop`` of ``multiply`` + ``Accum add`` over shared-memory loads, then the
micro-tile ``Write``s).  The reference lowers that IR to CUDA-core FFMAs with
a cp.async ring (``stmt_cpasync_copy`` ``compile.py:1754-1772``, full unroll
``:1882-1928``, FMA contraction ``:2250-2264``).  This template keeps the
IR's CTA -> output-tile assignment and computes each tile with:

* TMA (``cp.async.bulk.tensor.2d``, each CTA copying for itself) loading 128-byte-swizzled
  A and B k-slices into an S-stage shared-memory ring, one elected thread,
  completion counted on an mbarrier (``complete_tx``);
* one elected thread issuing ``tcgen05.mma.cta_group::1.kind::f16`` (bf16
  inputs, f32 accumulate; M=128, N=BN, K=16 per instruction) with the
  accumulator in tensor memory (``tcgen05.alloc``), each stage released back
  to the producer by ``tcgen05.commit`` on its ``empty`` mbarrier;
* all warps draining TMEM with ``tcgen05.ld.32x32b.x32`` (warp w reads lanes
  32*(w%4)..+31, i.e. output rows) and writing 32-byte ``st.global.v8`` rows.

A is K-major ([M,K] row-major) and B MN-major ([K,N] row-major), both with
a 128-byte swizzle; the shared-memory matrix descriptors follow the UMMA
canonical layouts (K-major: 8-row groups 1024 B apart; MN-major 16-bit:
64-element N blocks ``BK*128`` B apart, 8-row K groups 1024 B apart;
MN-major 32-bit (tf32): the 128-byte swizzle with 32-byte atoms, 32-element N
blocks ``BK*128`` B apart, 4-row K groups 512 B apart).

fp32 operands take the 3xTF32 route: converter warps write the low part of
each landed k-slice next to it in shared memory and the MMA thread issues
``kind::tf32`` MMAs for lo*hi, hi*lo and hi*hi.  The high part is the raw
f32 slice itself: the tensor core reads the top 19 bits of a 32-bit tf32
element, so hi = x with its 13 low mantissa bits dropped, and the converters
write only lo = x - hi (``tf32_lo_trunc``, exact in f32).  The lo*lo term and
the tensor core's truncation of lo, each below 2^-20 relative, are the only
losses of the split.

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
    (2 = 128-byte swizzle with 16-byte atoms, 1 = 128-byte swizzle with
    32-byte atoms); the start address (>>4) is added at run time."""
    return ((lbo >> 4) << 16) | ((sbo >> 4) << 32) | (1 << 46) | (swizzle_code << 61)


def idesc_mma(M: int, N: int, b_mn_major: bool, tf32: bool = False) -> int:
    """Instruction descriptor of ``tcgen05.mma`` (kind::f16 / kind::tf32): f32
    accumulator (bits 4-5 = 1), A and B format at bits 7-9 / 10-12 (1 = bf16,
    2 = tf32), A K-major, B major-ness at bit 16, N>>3 at bits 17-22, M>>4 at
    bits 24-28."""
    fmt = 2 if tf32 else 1
    return (1 << 4) | (fmt << 7) | (fmt << 10) | (int(b_mn_major) << 16) | ((N >> 3) << 17) \
        | ((M >> 4) << 24)


# 3xTF32 high parts: the raw slice (True: converters write lo only) or
# cvt.rna-rounded copies written back in place (False)
TF32_HI_RAW = True


def tf32_lo_trunc(k, x):
    """Low tf32 parts of four f32 registers for a high part that the tensor
    core takes from the raw element (its top 19 bits): lo = x - (x with the
    13 low mantissa bits cleared), exact in f32.  On the BASELINE 3xTF32 GEMM
    this saves the converters a third of their shared-memory traffic (no
    high-part stores): 261.5-269.1 TFLOP/s against 256.5-257.0 with
    ``tf32_split``, and the same error against float64 (normwise 2.93e-5
    against 2.87e-5 at 1024 x 1024 x 4096; a tensor core that rounded the raw
    element instead would show a bias of about 2^-11)."""
    lo = k.regs("r", 4)
    for j in range(4):
        t = k.reg("r")
        k(f"and.b32 {t}, {x[j]}, -8192;")
        k(f"sub.rn.f32 {lo[j]}, {x[j]}, {t};")
    return lo


def tf32_split(k, x):
    """Split four f32 registers into tf32 high parts ``cvt.rna.tf32(x)`` and
    low parts ``x - hi`` (exact in f32, left unrounded: the tensor core keeps
    about 11 significant bits of it, so hi + lo carries x to within 2^-21
    relative; the dropped lo*lo product is smaller still).  Measured on the
    BASELINE 3xTF32 GEMM: 240 TFLOP/s, against 232 with lo rounded by a
    second cvt and 216 with hi formed by masking (scalar or packed pairs)."""
    hi, lo = k.regs("r", 4), k.regs("r", 4)
    for j in range(4):
        k(f"cvt.rna.tf32.f32 {hi[j]}, {x[j]};")
        k(f"sub.rn.f32 {lo[j]}, {x[j]}, {hi[j]};")
    return hi, lo


class GemmTemplate:
    name = "gemm"
    # bf16 128x256 tiles whose M-neighbours can pair up run as CTA pairs
    # (templates/gemm_pair.py); False forces the single-CTA kernel
    PAIR = True
    # pair kernels whose ring fits 4+ stages (one CTA per SM) run persistent
    # with a double-buffered accumulator (templates/gemm_persistent.py)
    PERSISTENT = True

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "GemmTemplate":
        from .gemm_small import meta_only
        if meta_only():
            raise TemplateMismatch("meta-only launch requested (EMMY_META_ONLY): no tensor maps")
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
        if dts == {"bf16"}:
            mode = "bf16"
        elif dts == {"f32"}:
            mode = "tf32x3"
        else:
            raise TemplateMismatch(f"operand dtypes {dts}")
        threads = ctx.threads
        if ctx.block != (threads, 1, 1) or threads != 256:
            raise TemplateMismatch("tcgen05 template runs 256-thread CTAs")
        if ctx.grid[0] * ctx.grid[1] * ctx.grid[2] != ext["a0_b"] * ext["a1_b"]:
            raise TemplateMismatch("grid is not one CTA per output tile")
        self = cls()
        self.mode = mode
        self.esize = 2 if mode == "bf16" else 4
        self.BK = 128 // self.esize          # one 128-byte swizzle row of K per stage
        self.box_n = 128 // self.esize       # B loaded as 128-byte-wide column boxes
        if BM != 128 or BN % self.box_n or not 64 <= BN <= 256 or BN % 16 or K % self.BK:
            raise TemplateMismatch(f"tile {BM}x{BN}, K={K} outside the tcgen05 shapes")
        self.ctx, self.A, self.B, self.C = ctx, A, B, C
        self.M, self.N, self.K, self.BM, self.BN = M, N, K, BM, BN
        raw = (BM * self.BK + self.BK * BN) * self.esize
        # 3xTF32 keeps a low-part copy of each operand slice next to it
        stage = raw * (2 if mode == "tf32x3" else 1)
        self.stage_bytes = stage
        avail = min(ctx.smem_bytes, SMEM_LIMIT) - 1024 - 256
        self.S = min(6, avail // stage)
        if self.S < 2:
            raise TemplateMismatch("meta smem_bytes too small for a 2-stage ring")
        self.NB = ext["a1_b"]
        self.hw_trunc = False
        from .gemm_pair import PAIR_STAGE, pair_stages
        # 3xTF32 pairs keep each CTA's raw slice and its low parts: 64 KiB
        self.pair_S = pair_stages(ctx.smem_bytes, SMEM_LIMIT,
                                  PAIR_STAGE * (2 if mode == "tf32x3" else 1))
        self.pair = (cls.PAIR and BM == 128 and BN == 256
                     and (M // BM) % 2 == 0 and self.pair_S >= 2
                     and tuple(ctx.grid[1:]) == (1, 1))
        return self

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        if self.pair and (self.mode == "bf16" or type(self).PERSISTENT):
            from .gemm_persistent import PERSISTENT_MIN_STAGES, emit_pair_persistent
            # 3xTF32 pair stages are 64 KiB: two already mean one CTA per SM
            if type(self).PERSISTENT and (self.pair_S >= PERSISTENT_MIN_STAGES
                                          or self.mode == "tf32x3"):
                return emit_pair_persistent(self)
            from .gemm_pair import emit_pair
            return emit_pair(self)
        ctx = self.ctx
        BM, BN, BK, S, K = self.BM, self.BN, self.BK, self.S, self.K
        es = self.esize
        tf32 = self.mode == "tf32x3"
        KT = K // BK
        SA = BM * BK * es                # A slice bytes (16 KiB)
        SB = BK * BN * es                # B slice bytes
        RAW = SA + SB
        STG = self.stage_bytes           # raw (+ low parts) per stage
        BOXN = self.box_n
        NBOX = BN // BOXN
        KMMA = 32 // es                  # K per tcgen05.mma (32 bytes of K)
        tm_dtype = 9 if not tf32 else 7  # CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 / FLOAT32
        params = ctx.params() + [("tmapA", ".align 64 .b8", "[128]"),
                                 ("tmapB", ".align 64 .b8", "[128]")]
        k = Kernel(ctx.entry, params)
        k.maxntid = (256, 1, 1)
        k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
        k.decl(".global .align 4 .u32 __emmy_status;")
        # host-built tensor maps (innermost dimension first)
        k.directive(f"tmap tmapA buf={self.A} dtype={tm_dtype} dims={K},{self.M} "
                    f"strides={K * es} box={BK},{BM} swizzle=3")
        # MN-major 32-bit operands need the 128-byte swizzle with 32-byte atoms
        # (4-row K groups); 16-bit ones use the plain 128-byte swizzle
        b_swz = 4 if tf32 else 3
        k.directive(f"tmap tmapB buf={self.B} dtype={tm_dtype} dims={self.N},{K} "
                    f"strides={self.N * es} box={BOXN},{BK} swizzle={b_swz}")
        k.comment(f"emmy-b200 template: tcgen05 gemm {self.mode} M={self.M} N={self.N} K={K} "
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
        # shared memory (1024-aligned base): S stages of [A | B (| A_lo | B_lo)],
        # then mbarriers: full[S], empty[S], conv[S] (3xTF32), accum, tmem slot
        raw = k.reg("r")
        k(f"mov.u32 {raw}, __emmy_smem;")
        ring = k.reg("r")
        k(f"add.u32 {ring}, {raw}, 1023;")
        k(f"and.b32 {ring}, {ring}, -1024;")
        bars = k.reg("r")
        k(f"add.u32 {bars}, {ring}, {S * STG};")
        nb = 3 * S if tf32 else 2 * S
        accb = k.reg("r")
        k(f"add.u32 {accb}, {bars}, {8 * nb};")
        tslot = k.reg("r")
        k(f"add.u32 {tslot}, {accb}, 8;")
        status = k.reg("rd")
        k(f"mov.u64 {status}, __emmy_status;")
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip_init = k.label("SKIP_INIT")
        k(f"@!{p0} bra {skip_init};")
        for s in range(2 * S):
            k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], 1;")
        for s in range(2 * S, nb):       # conv[s]: the 128 converter threads arrive
            k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * s}], 128;")
        k(f"mbarrier.init.shared::cta.b64 [{accb}], 1;")
        k("fence.mbarrier_init.release.cluster;")
        k(f"prefetch.tensormap [{ta}];")
        k(f"prefetch.tensormap [{tb}];")
        k.mark(skip_init)
        pw1 = k.reg("p")
        k(f"setp.eq.u32 {pw1}, {warp}, 1;")
        skip_alloc = k.label("SKIP_ALLOC")
        k(f"@!{pw1} bra {skip_alloc};")
        ncols = max(32, 1 << (BN - 1).bit_length())
        k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{tslot}], {ncols};")
        k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
        k.mark(skip_alloc)
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
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
            self._advance(k, st, ph, S)
            k(f"add.u32 {kt}, {kt}, 1;")
            pl = k.reg("p")
            k(f"setp.lt.u32 {pl}, {kt}, {KT};")
            k(f"@{pl} bra {top};")

        # ---------------- producer: warp 0, lane 0 ----------------
        pprod = k.reg("p")
        k(f"setp.eq.u32 {pprod}, {warp}, 0;")
        k(f"and.pred {pprod}, {pprod}, {pl0};")
        end_prod = k.label("END_PROD")
        k(f"@!{pprod} bra {end_prod};")
        top = loop_head("PROD")
        par = k.reg("r")
        k(f"xor.b32 {par}, {ph}, 1;")
        self._wait(k, bar_addr(1, st), par, status, 1, end_prod)
        fb = bar_addr(0, st)
        k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {RAW};")
        kc = k.reg("r")
        k(f"mul.lo.u32 {kc}, {kt}, {BK};")
        da = stage_base(st)
        k(f"cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
          f"[{da}], [{ta}, {{{kc}, {m0}}}], [{fb}];")
        for i in range(NBOX):
            nx = k.reg("r")
            k(f"add.u32 {nx}, {n0}, {BOXN * i};")
            db = k.reg("r")
            k(f"add.u32 {db}, {da}, {SA + i * BK * 128};")
            k(f"cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
              f"[{db}], [{tb}, {{{nx}, {kc}}}], [{fb}];")
        loop_tail(top)
        k.mark(end_prod)

        # ---------------- 3xTF32 converters: warps 4-7 ----------------
        if tf32:
            self._converters(k, warp, tid, bar_addr, stage_base, loop_head, loop_tail, status,
                             RAW, st, ph)

        # ---------------- MMA issuer: warp 1, lane 0 ----------------
        pmma = k.reg("p")
        k(f"setp.eq.u32 {pmma}, {warp}, 1;")
        k(f"and.pred {pmma}, {pmma}, {pl0};")
        end_mma = k.label("END_MMA")
        k(f"@!{pmma} bra {end_mma};")
        idesc = k.reg("r")
        k(f"mov.u32 {idesc}, {idesc_mma(BM, BN, True, tf32)};")
        hiA = _desc_hi(16, 1024)
        hiB = _desc_hi(BK * 128, 512, 1) if tf32 else _desc_hi(BK * 128, 1024)
        top2 = loop_head("MMA")
        self._wait(k, bar_addr(2 if tf32 else 0, st), ph, status, 2, end_mma)
        k("tcgen05.fence::after_thread_sync;")
        sb = stage_base(st)
        bad = k.reg("r")
        k(f"add.u32 {bad}, {sb}, {SA};")
        adesc = self._desc(k, sb, hiA)
        bdesc = self._desc(k, bad, hiB)
        if tf32:
            lad = k.reg("r")
            k(f"add.u32 {lad}, {sb}, {RAW};")
            lbd = k.reg("r")
            k(f"add.u32 {lbd}, {sb}, {RAW + SA};")
            ldesc_a = self._desc(k, lad, hiA)
            ldesc_b = self._desc(k, lbd, hiB)
        pacc = k.reg("p")
        k(f"setp.ne.u32 {pacc}, {kt}, 0;")
        ptrue = k.reg("p")
        k(f"setp.eq.u32 {ptrue}, 0, 0;")
        kind_ = "tf32" if tf32 else "f16"
        first = True
        for kk in range(BK // KMMA):
            ao, bo = kk * 2, kk * KMMA * 8   # +32 B along K (A); +KMMA rows of 128 B (B)
            pairs = [(adesc, bdesc)]
            if tf32:   # small terms first: lo*hi + hi*lo, then hi*hi
                pairs = [(ldesc_a, bdesc), (adesc, ldesc_b), (adesc, bdesc)]
            for da_, db_ in pairs:
                ad = k.reg("rd")
                k(f"add.s64 {ad}, {da_}, {ao};")
                bd = k.reg("rd")
                k(f"add.s64 {bd}, {db_}, {bo};")
                pa = pacc if first else ptrue
                first = False
                k(f"tcgen05.mma.cta_group::1.kind::{kind_} [{tmem}], {ad}, {bd}, {idesc}, {pa};")
        k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
          f"[{bar_addr(1, st)}];")
        loop_tail(top2)
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
        k(f"shl.b32 {taddr}, {q}, 21;")              # (32*q) << 16: TMEM lane field
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
        chunk = 32 if half % 32 == 0 else 16 if half % 16 == 0 else 8
        for c in range(half // chunk):
            regs = k.regs("r", chunk)
            ta2 = k.reg("r")
            k(f"add.u32 {ta2}, {taddr}, {chunk * c};")
            k(f"tcgen05.ld.sync.aligned.32x32b.x{chunk}.b32 {{{', '.join(regs)}}}, [{ta2}];")
            k("tcgen05.wait::ld.sync.aligned;")
            for v in range(chunk // 8):
                k(f"st.global.v8.b32 [{cptr}+{4 * chunk * c + 32 * v}], "
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
        k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {ncols};")
        k.mark(end)
        k("ret;")
        return k.render()

    def _converters(self, k, warp, tid, bar_addr, stage_base, loop_head, loop_tail, status,
                    RAW, st, ph):
        """Warps 4-7 split every landed stage for 3xTF32: for each f32 x of
        the A and B slices, lo goes into the stage's low-part area (the same
        swizzled layout, so the same descriptors apply); the high part is x
        itself (``tf32_lo_trunc``), or with ``TF32_HI_RAW`` off a rounded copy
        written back in place (``tf32_split``).  Then
        ``fence.proxy.async`` makes the generic-proxy stores visible to the
        tensor core's async-proxy reads before the conv[s] arrive."""
        pc = k.reg("p")
        k(f"setp.ge.u32 {pc}, {warp}, 4;")
        end_conv = k.label("END_CONV")
        k(f"@!{pc} bra {end_conv};")
        ct = k.reg("r")
        k(f"sub.u32 {ct}, {tid}, 128;")               # converter thread 0..127
        off0 = k.reg("r")
        k(f"shl.b32 {off0}, {ct}, 4;")                # 16 bytes per thread per pass
        top = loop_head("CONV")
        self._wait(k, bar_addr(0, st), ph, status, 4, end_conv)
        sb = stage_base(st)
        a0 = k.reg("r")
        k(f"add.u32 {a0}, {sb}, {off0};")
        per = RAW // (16 * 128)
        for i in range(per):
            x = k.regs("r", 4)
            ad = f"{a0}+{i * 2048}" if i else a0
            k(f"ld.shared.v4.b32 {{{', '.join(x)}}}, [{ad}];")
            if TF32_HI_RAW:
                lo = tf32_lo_trunc(k, x)
            else:
                hi, lo = tf32_split(k, x)
                k(f"st.shared.v4.b32 [{ad}], {{{', '.join(hi)}}};")
            k(f"st.shared.v4.b32 [{a0}+{RAW + i * 2048}], {{{', '.join(lo)}}};")
        k("fence.proxy.async.shared::cta;")
        k(f"mbarrier.arrive.shared::cta.b64 _, [{bar_addr(2, st)}];")
        loop_tail(top)
        k.mark(end_conv)

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
    def _wait(k, bar, parity, status, code, fail_label, sem=""):
        """Spin on ``mbarrier.try_wait.parity`` for at most WAIT_NS of
        %globaltimer; on expiry store ``code`` to ``__emmy_status`` and jump
        to ``fail_label``.  ``sem`` (e.g. ``.acquire.cluster``) widens the
        wait's acquire to the cluster for arrivals from the peer CTA.  The first try runs before the clock is read: a
        %globaltimer read costs hundreds of cycles, which would otherwise sit
        on the path of every wait that succeeds at once."""
        p = k.reg("p")
        top, ok = k.label("WAIT"), k.label("WAIT_OK")
        k(f"mbarrier.try_wait.parity{sem}.shared::cta.b64 {p}, [{bar}], {parity};")
        k(f"@{p} bra {ok};")
        t0 = k.reg("rd")
        k(f"mov.u64 {t0}, %globaltimer;")
        k.mark(top)
        k(f"mbarrier.try_wait.parity{sem}.shared::cta.b64 {p}, [{bar}], {parity};")
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

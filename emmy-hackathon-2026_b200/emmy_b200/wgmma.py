"""The warpgroup tensor-core statements (``wgmma``) mapped onto tcgen05.

The Kernel IR vocabulary defines, and no reference IR uses, the Hopper
warpgroup statements (reference ``TASK.md:164-172``): ``WgmmaDescriptor``
builds a shared-memory matrix descriptor, ``WgmmaMma`` issues one
asynchronous ``m64nNk16`` product of a warpgroup into its C fragments (in
registers), ``WgmmaFence`` / ``WgmmaCommit`` / ``WgmmaWait`` order, group and
wait for them.  ``wgmma`` is an sm_90a instruction; sm_100a has
``tcgen05.mma``, which one thread issues into tensor memory.  This module
keeps the statements' meaning on that machine:

* each warpgroup's accumulators (one per distinct ``c_frags``) live in tensor
  memory as M = 64 tiles, rows 16w..16w+15 of the tile in TMEM lanes
  32w..32w+15 -- the lanes warp w of the warpgroup can reach, read and written
  with ``tcgen05.ld/st .16x256b``, whose per-thread element order is the
  register order of the wgmma accumulator (the m16n8 C fragment per 8
  columns).  ``c_frags`` are those C fragments: a tuple of N / 8 fragment
  references, or one ``RegFragment`` array of N / 8 cells;
* registers stay the program's copy of an accumulator: a ``WgmmaMma`` whose
  registers are current (nothing issued on them since the last wait) first
  writes them into tensor memory, so ``scale_d`` = 1 accumulates onto what the
  program holds; ``WgmmaWait`` reads every accumulator issued on since the last
  wait back into its registers (a per-accumulator flag, uniform in the
  warpgroup, says which);
* the product is issued by the warpgroup's first thread as
  ``tcgen05.mma.cta_group::1`` (M = 64, the IR's N, A / B major-ness from
  ``trans_a`` / ``trans_b``, ``scale_d`` as the accumulate predicate) after a
  warpgroup barrier; ``WgmmaCommit`` commits the warpgroup's products to one of
  ``RING`` mbarriers, ``WgmmaWait(n)`` waits for all committed groups (at most
  n pending is implied) with bounded waits (status 8 on expiry);
* ``WgmmaDescriptor`` encodes the tcgen05 form of the descriptor: start
  address of ``smem[smem_index]``, ``lbo_bytes`` / ``sbo_bytes``, version 1,
  the swizzle (``NONE``, ``128B``, ``64B``, ``32B``, or Hopper's codes 1 / 2 /
  3 for them);
* shared memory written by threads reaches the tensor core through
  ``fence.proxy.async``: the lowering emits one before every CTA barrier of a
  kernel that uses these statements, and ``WgmmaFence`` is that fence plus a
  warpgroup barrier.

* an A operand in registers (``a_frag``: the warp's 16 rows of the 64 x 16
  A tile as an m16n8k16 A fragment, bf16 or f16) is written by the
  warpgroup into a 2 KiB shared-memory slot in the unswizzled K-major layout
  (8x8 core matrices, LBO 128 B along K, SBO 256 B along M) and read through
  a descriptor; the slot is reused only after the product that read it has
  completed (its own commit and bounded wait), so such products run one at a
  time.

Limits (exit 1, ``unsupported construct``): a one-dimensional CTA of whole
warpgroups with every thread a cell; at most 512 tensor-memory columns over
all warpgroups' accumulators; a register A operand of tf32.
"""
from __future__ import annotations

import re

from .analysis import kind, walk
from .ir import dim

RING = 8
_SWZ = {None: 0, "NONE": 0, "none": 0, 0: 0, "128B": 2, "B128": 2, "SWIZZLE_128B": 2, 1: 2,
        "64B": 4, "B64": 4, "SWIZZLE_64B": 4, 2: 4, "32B": 6, "B32": 6, "SWIZZLE_32B": 6, 3: 6}
_FMT = {"f16": 0, "bf16": 1, "tf32": 2}


def _wg_shape(s):
    if isinstance(s, str):
        m = re.fullmatch(r"m(\d+)n(\d+)k(\d+)", s)
        if not m:
            raise NotImplementedError(f"wgmma shape {s!r}")
        t = tuple(int(x) for x in m.groups())
    else:
        t = tuple(int(x) for x in s)
    M, N, K = t
    if M != 64 or N % 8 or not 8 <= N <= 256 or K not in (8, 16):
        raise NotImplementedError(f"wgmma shape m{M}n{N}k{K}")
    return t


def _key(c_frags) -> tuple:
    return tuple(c_frags) if isinstance(c_frags, tuple) else (str(c_frags),)


def desc_hi(lbo: int, sbo: int, swz: int) -> int:
    """Constant bits of a tcgen05 shared-memory descriptor: LBO >> 4 at 16,
    SBO >> 4 at 32, version 1 at 46, swizzle at 61."""
    return ((lbo >> 4) << 16) | ((sbo >> 4) << 32) | (1 << 46) | (swz << 61)


def idesc(M: int, N: int, fmt: int, a_mn: bool, b_mn: bool) -> int:
    """tcgen05 instruction descriptor, f32 accumulator."""
    return (1 << 4) | (fmt << 7) | (fmt << 10) | (int(a_mn) << 15) | (int(b_mn) << 16) \
        | ((N >> 3) << 17) | ((M >> 4) << 24)


class WgmmaLowering:
    """Mixin of ``GenericLowering``: set-up and teardown around the body, and
    the ``s_Wgmma*`` statement methods."""

    _wg = None

    # ------------------------------------------------------------ set-up
    def _wg_cells(self, c_frags):
        """The C fragment cells of an accumulator, in column order."""
        if isinstance(c_frags, tuple):
            return [self._ref(r) for r in c_frags]
        f = self._frag_state().get(str(c_frags))
        if f is None:
            raise NotImplementedError(f"wgmma accumulator {c_frags} has no RegFragment")
        return [(f, cell) for cell in f.cells]

    def _wg_begin(self, tile):
        muls = [s for s in walk(tile.body) if kind(s) == "WgmmaMma"]
        if not muls:
            return
        ctx, k = self.ctx, self.k
        bx, by, bz = ctx.block
        ncells = 1
        for a in tile.axes:
            ncells *= dim(a.extent)
        if by * bz != 1 or bx % 128 or ncells != ctx.total_threads or \
                int(getattr(tile, "aux_threads", 0) or 0):
            raise NotImplementedError("wgmma needs a one-dimensional CTA of whole warpgroups "
                                      "with every thread a cell")
        widths: dict = {}
        cfr: dict = {}
        areg = False
        for s in muls:
            if getattr(s, "a_frag", None):
                areg = True
                if _wg_shape(s.shape)[2] != 16:
                    raise NotImplementedError("wgmma register A operand of tf32")
            n = _wg_shape(s.shape)[1]
            key = _key(s.c_frags)
            cfr[key] = s.c_frags
            if widths.setdefault(key, n) != n:
                raise NotImplementedError("one wgmma accumulator used with two widths")
        offs, col = {}, 0
        for key, n in widths.items():
            offs[key] = col
            col += n
        nwg = bx // 128
        need = nwg * col
        ncols = 32
        while ncols < need:
            ncols *= 2
        if ncols > 512:
            raise NotImplementedError(f"wgmma accumulators need {need} tensor-memory columns")
        k.decl(f".shared .align 8 .b8 __emmy_wg_bar[{8 * (RING + 1) * nwg}];")
        if areg:
            k.decl(f".shared .align 128 .b8 __emmy_wg_astage[{2048 * nwg}];")
        k.decl(".shared .align 4 .b8 __emmy_wg_tmem[4];")
        tid, warp = self.tid_x, self.ints["warp"]
        bb = k.reg("r")
        k(f"mov.u32 {bb}, __emmy_wg_bar;")
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip = k.label("WG_INIT")
        k(f"@!{p0} bra {skip};")
        for i in range((RING + 1) * nwg):
            k(f"mbarrier.init.shared::cta.b64 [{bb}+{8 * i}], 1;")
        k("fence.mbarrier_init.release.cluster;")
        k.mark(skip)
        pw = k.reg("p")
        k(f"setp.eq.u32 {pw}, {warp}, 0;")
        skip2 = k.label("WG_ALLOC")
        k(f"@!{pw} bra {skip2};")
        slot = k.reg("r")
        k(f"mov.u32 {slot}, __emmy_wg_tmem;")
        k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{slot}], {ncols};")
        k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
        k.mark(skip2)
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
        k("tcgen05.fence::after_thread_sync;")
        tm = k.reg("r")
        k(f"ld.shared.u32 {tm}, [__emmy_wg_tmem];")
        wg = k.reg("r")
        k(f"shr.u32 {wg}, {warp}, 2;")
        mytm = k.reg("r")                    # this warpgroup's first column
        k(f"mad.lo.s32 {mytm}, {wg}, {col}, {tm};")
        lb = k.reg("r")                      # + this warp's lane quarter
        k(f"and.b32 {lb}, {warp}, 3;")
        k(f"shl.b32 {lb}, {lb}, 21;")
        k(f"add.s32 {lb}, {lb}, {mytm};")
        bars = k.reg("r")                    # RING group barriers, then the A-slot barrier
        k(f"mad.lo.s32 {bars}, {wg}, {8 * (RING + 1)}, {bb};")
        bid = k.reg("r")
        k(f"add.s32 {bid}, {wg}, 8;")
        el = k.reg("p")
        t7 = k.reg("r")
        k(f"and.b32 {t7}, {tid}, 127;")
        k(f"setp.eq.u32 {el}, {t7}, 0;")
        c, w, unc = k.reg("r"), k.reg("r"), k.reg("r")
        abusy, aph = k.reg("r"), k.reg("r")
        for r in (c, w, unc, abusy, aph):
            k(f"mov.u32 {r}, 0;")
        astage = None
        if areg:
            astage = k.reg("r")
            k(f"mov.u32 {astage}, __emmy_wg_astage;")
            k(f"mad.lo.s32 {astage}, {wg}, 2048, {astage};")
        auth = {}
        for key in widths:
            auth[key] = k.reg("r")
            k(f"mov.u32 {auth[key]}, 1;")
        self._wg = {"tm": tm, "mytm": mytm, "lb": lb, "bars": bars, "bid": bid, "el": el,
                    "c": c, "w": w, "unc": unc, "auth": auth, "offs": offs, "ncols": ncols,
                    "cfr": cfr, "abusy": abusy, "aph": aph, "astage": astage}
        self.wg_descs = {}

    def _wg_end(self):
        wg = self._wg
        if wg is None:
            return
        k = self.k
        self._wg_wait_all()
        if wg["astage"] is not None:
            self._wg_slot_free()
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
        k("tcgen05.fence::after_thread_sync;")
        pw = k.reg("p")
        k(f"setp.eq.u32 {pw}, {self.ints['warp']}, 0;")
        skip = k.label("WG_FREE")
        k(f"@!{pw} bra {skip};")
        k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {wg['tm']}, {wg['ncols']};")
        k.mark(skip)

    # ------------------------------------------------------------ helpers
    def _wg_need(self):
        if self._wg is None:
            raise NotImplementedError("wgmma statement outside a kernel that issues WgmmaMma")
        return self._wg

    def _wg_sync(self):
        """Warpgroup barrier with tcgen05 ordering on both sides."""
        wg, k = self._wg, self.k
        k("tcgen05.fence::before_thread_sync;")
        k(f"bar.sync {wg['bid']}, 128;")
        k("tcgen05.fence::after_thread_sync;")

    def _wg_wait_one(self):
        """Wait for committed group number w (mbarrier w % RING, parity of
        w / RING), then w += 1."""
        wg, k = self._wg, self.k
        slot = k.reg("r")
        k(f"rem.u32 {slot}, {wg['w']}, {RING};")
        a = k.reg("r")
        k(f"mad.lo.s32 {a}, {slot}, 8, {wg['bars']};")
        par = k.reg("r")
        k(f"div.u32 {par}, {wg['w']}, {RING};")
        k(f"and.b32 {par}, {par}, 1;")
        self.bounded_parity_wait(a, par)
        k(f"add.u32 {wg['w']}, {wg['w']}, 1;")

    def _wg_slot_free(self):
        """Wait (bounded) for the product that last read the A slot."""
        wg, k = self._wg, self.k
        pb = k.reg("p")
        k(f"setp.ne.u32 {pb}, {wg['abusy']}, 0;")
        skip = k.label("WG_SLOT")
        k(f"@!{pb} bra {skip};")
        a = k.reg("r")
        k(f"add.s32 {a}, {wg['bars']}, {8 * RING};")
        self.bounded_parity_wait(a, wg["aph"])
        k(f"xor.b32 {wg['aph']}, {wg['aph']}, 1;")
        k(f"mov.u32 {wg['abusy']}, 0;")
        k.mark(skip)
        k("tcgen05.fence::after_thread_sync;")

    def _wg_stage_a(self, ref):
        """The warp's A fragment (rows 16 w.., 16 k) into the A slot, K-major
        without swizzle: element (m, k) at (m/8)*256 + (k/8)*128 + (m%8)*16 +
        (k%8)*2 bytes.  Returns the slot's descriptor."""
        wg, k = self._wg, self.k
        f, regs = self._ref(ref)
        if f.role != "a" or f.dt not in ("bf16", "f16") or f.shape[2] != 16:
            raise NotImplementedError("wgmma a_frag must be a 16-bit m16n8k16 A fragment")
        self._wg_slot_free()
        g, t = self._lane_gt()
        w4 = k.reg("r")
        k(f"and.b32 {w4}, {self.ints['warp']}, 3;")
        # rows 16 w4 + g (+8), k = 2t (+8): byte = (2 w4 + h) * 256 + kh * 128 + g * 16 + t * 4
        base = k.reg("r")
        k(f"mad.lo.s32 {base}, {w4}, 512, {wg['astage']};")
        k(f"mad.lo.s32 {base}, {g}, 16, {base};")
        k(f"mad.lo.s32 {base}, {t}, 4, {base};")
        for r, (dh, kh) in zip(regs, [(0, 0), (1, 0), (0, 1), (1, 1)]):
            k(f"st.shared.b32 [{base}+{dh * 256 + kh * 128}], {r};")
        k("fence.proxy.async.shared::cta;")
        d = k.reg("rd")
        k(f"cvt.u64.u32 {d}, {wg['astage']};")
        k(f"shr.u64 {d}, {d}, 4;")
        k(f"and.b64 {d}, {d}, 16383;")
        k(f"or.b64 {d}, {d}, {desc_hi(128, 256, 0)};")
        return d

    def _wg_commit(self):
        wg, k = self._wg, self.k
        # a full ring: the oldest group must complete before its barrier is reused
        full = k.reg("p")
        d = k.reg("r")
        k(f"sub.u32 {d}, {wg['c']}, {wg['w']};")
        k(f"setp.lt.u32 {full}, {d}, {RING};")
        skip = k.label("WG_ROOM")
        k(f"@{full} bra {skip};")
        self._wg_wait_one()
        k.mark(skip)
        slot = k.reg("r")
        k(f"rem.u32 {slot}, {wg['c']}, {RING};")
        a = k.reg("r")
        k(f"mad.lo.s32 {a}, {slot}, 8, {wg['bars']};")
        skip2 = k.label("WG_COMMIT")
        k(f"@!{wg['el']} bra {skip2};")
        k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{a}];")
        k.mark(skip2)
        k(f"add.u32 {wg['c']}, {wg['c']}, 1;")
        k(f"mov.u32 {wg['unc']}, 0;")

    def _wg_wait_all(self):
        wg, k = self._wg, self.k
        pu = k.reg("p")
        k(f"setp.ne.u32 {pu}, {wg['unc']}, 0;")
        skip = k.label("WG_NOUNC")
        k(f"@!{pu} bra {skip};")
        self._wg_commit()
        k.mark(skip)
        top, end = k.label("WG_WAIT"), k.label("WG_WAITED")
        k.mark(top)
        pd = k.reg("p")
        k(f"setp.ge.u32 {pd}, {wg['w']}, {wg['c']};")
        k(f"@{pd} bra {end};")
        self._wg_wait_one()
        k(f"bra.uni {top};")
        k.mark(end)
        k("tcgen05.fence::after_thread_sync;")

    def _wg_addr(self, key, i) -> str:
        """This warp's TMEM address of 8-column block i of accumulator key."""
        wg, k = self._wg, self.k
        a = k.reg("r")
        k(f"add.s32 {a}, {wg['lb']}, {wg['offs'][key] + 8 * i};")
        return a

    # ------------------------------------------------------------ statements
    def s_WgmmaDescriptor(self, s):
        k = self.k
        self._wg_need()
        swz = s.swizzle
        if isinstance(swz, str):
            swz = swz.strip()
        if swz not in _SWZ:
            raise NotImplementedError(f"wgmma descriptor swizzle {s.swizzle!r}")
        lbo, sbo = self._literal_int(s.lbo_bytes), self._literal_int(s.sbo_bytes)
        if lbo is None or sbo is None or lbo % 16 or sbo % 16:
            raise NotImplementedError("wgmma descriptor offsets must be literal multiples of 16")
        if s.smem not in self.smem:
            raise NotImplementedError(f"wgmma descriptor of {s.smem}: not shared memory")
        addr = self.saddr(s.smem, self.flat(tuple(s.smem_index), self.shape_of(s.smem)))
        d = k.reg("rd")
        k(f"cvt.u64.u32 {d}, {addr};")
        k(f"shr.u64 {d}, {d}, 4;")
        k(f"and.b64 {d}, {d}, 16383;")
        k(f"or.b64 {d}, {d}, {desc_hi(lbo, sbo, _SWZ[swz])};")
        self.wg_descs[s.name] = d

    def s_WgmmaFence(self, s):
        self._wg_need()
        self.k("fence.proxy.async.shared::cta;")
        self._wg_sync()

    def s_WgmmaMma(self, s):
        wg, k = self._wg_need(), self.k
        M, N, K = _wg_shape(s.shape)
        key = _key(s.c_frags)
        cells = self._wg_cells(s.c_frags)
        if len(cells) != N // 8 or any(f.role != "c" or f.dt != "f32" for f, _ in cells):
            raise NotImplementedError(f"wgmma m64n{N}: c_frags must be {N // 8} f32 C fragments")
        ab = getattr(s.ab_dtype, "name", s.ab_dtype) or "bf16"
        ab = {"bfloat16": "bf16", "float16": "f16"}.get(str(ab), str(ab))
        if ab not in _FMT or (ab == "tf32") != (K == 8):
            raise NotImplementedError(f"wgmma {ab} k{K}")
        areg = bool(getattr(s, "a_frag", None))
        for nm in ((s.b_desc,) if areg else (s.a_desc, s.b_desc)):
            if nm not in self.wg_descs:
                raise NotImplementedError(f"wgmma operand descriptor {nm!r} not built")
        if areg and (s.trans_a or ab == "tf32"):
            raise NotImplementedError("wgmma register A operand: 16-bit, K-major")
        adesc = self._wg_stage_a(s.a_frag) if areg else self.wg_descs[s.a_desc]
        auth = wg["auth"][key]
        # the registers are the current accumulator: write them to tensor memory
        pa = k.reg("p")
        k(f"setp.ne.u32 {pa}, {auth}, 0;")
        skip = k.label("WG_NOST")
        k(f"@!{pa} bra {skip};")
        for i, (f, regs) in enumerate(cells):
            k(f"tcgen05.st.sync.aligned.16x256b.x1.b32 [{self._wg_addr(key, i)}], "
              f"{{{', '.join(regs)}}};")
        k("tcgen05.wait::st.sync.aligned;")
        k.mark(skip)
        self._wg_sync()
        sd = s.scale_d
        ps = k.reg("p")
        lit = self._literal_int(sd) if (sd is None or isinstance(sd, int) or
                                         kind(sd) == "Literal") else None
        if sd is None:
            lit = 1
        if lit is not None:
            k(f"setp.ne.u32 {ps}, {int(bool(lit))}, 0;")
        else:
            ps = self.pred(sd)
        idx = k.reg("r")
        k(f"mov.u32 {idx}, {idesc(M, N, _FMT[ab], bool(s.trans_a), bool(s.trans_b))};")
        d = k.reg("r")
        k(f"add.s32 {d}, {wg['mytm']}, {wg['offs'][key]};")
        skip2 = k.label("WG_ISSUE")
        k(f"@!{wg['el']} bra {skip2};")
        kd = "tf32" if ab == "tf32" else "f16"
        k(f"tcgen05.mma.cta_group::1.kind::{kd} [{d}], {adesc}, "
          f"{self.wg_descs[s.b_desc]}, {idx}, {ps};")
        if areg:
            # the slot is free again once this product completes
            sa = k.reg("r")
            k(f"add.s32 {sa}, {wg['bars']}, {8 * RING};")
            k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{sa}];")
        k.mark(skip2)
        if areg:
            k(f"mov.u32 {wg['abusy']}, 1;")
        k(f"mov.u32 {auth}, 0;")
        k(f"mov.u32 {wg['unc']}, 1;")

    def s_WgmmaCommit(self, s):
        self._wg_need()
        self._wg_commit()

    def s_WgmmaWait(self, s):
        wg, k = self._wg_need(), self.k
        self._wg_wait_all()
        for key, auth in wg["auth"].items():
            cells = self._wg_cells(wg["cfr"][key])
            pa = k.reg("p")
            k(f"setp.eq.u32 {pa}, {auth}, 0;")
            skip = k.label("WG_NOLD")
            k(f"@!{pa} bra {skip};")
            for i, (f, regs) in enumerate(cells):
                k(f"tcgen05.ld.sync.aligned.16x256b.x1.b32 {{{', '.join(regs)}}}, "
                  f"[{self._wg_addr(key, i)}];")
            k("tcgen05.wait::ld.sync.aligned;")
            k(f"mov.u32 {auth}, 1;")
            k.mark(skip)

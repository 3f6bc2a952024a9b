"""Matmul template with a meta-only launch: tcgen05 tiles fed by the CTA's own
threads instead of tensor maps.

The TMA kernels of :mod:`.gemm` take host-built tensor maps after the meta
``arg_order`` parameters; a launcher that passes exactly ``arg_order`` (the
reference's runner and its ctypes harness, ``tools/harness/gpu_run.py:82-89``)
cannot supply them.  This template's PTX takes the meta parameters and nothing
else, so it runs under any launcher of the reference's contract.  It accepts
Emmy's own matmul schedules -- the m01/m02 open problems and the corpus
``mm*`` IRs (reference ``problems/m01_matmul_512/*.ir.txt:1-37``): any CTA
tile up to 128 x 256, any CTA size from 32 threads, tiles cut off by the
matrix edge (``Cond(row < M)`` around ``% M`` stores) and split-K over a
leading Tile axis with atomic stores (``red.global.add``, the output zeroed
by ``zero_outputs``) -- and, when ``EMMY_META_ONLY=1`` makes the TMA
template decline, the benchmark's own matmul IRs.

Per CTA (the IR's CTA -> (k chunk, M tile, N tile) assignment, row-major over
the Tile's block axes):

* every thread stages 16-byte chunks of the A rows (K-major, as stored) and
  of the B columns (transposed on the way into K-major, four or eight
  scalar loads of a column per chunk, coalesced across the threads) into
  shared memory in the UMMA 128-byte-swizzle layout (the 16-byte chunk c of
  row r of an 8-row atom at chunk c ^ r), zero outside the matrix and past
  the CTA's K range; for fp32 operands the same threads also write the
  low tf32 parts lo = x - (x with its 13 low mantissa bits cleared) beside
  them (3xTF32, as :func:`.gemm.tf32_lo_trunc`);
* one thread issues ``tcgen05.mma.cta_group::1`` (M = 128, N = the tile
  width rounded up to 16; ``kind::tf32`` lo*hi, hi*lo, hi*hi or
  ``kind::f16``) into a TMEM accumulator and commits to the slab's
  mbarrier; two slab buffers alternate, so the threads stage slab s+1 while
  the tensor core works on slab s;
* the warps read the accumulator back with ``tcgen05.ld.32x32b`` (warp w:
  TMEM lanes 32 (w % 4) ..; warps with the same w % 4 split the columns)
  and store the CTA's in-bounds outputs (plain or atomic, as the IR writes).

Rows of the A operand beyond the tile (up to the MMA's 128) and columns beyond the tile
width only produce accumulator rows and columns that are never stored.
Every mbarrier wait is bounded by ``%globaltimer`` and reports through
``__emmy_status``.
"""
from __future__ import annotations

import os

from ..analysis import NotAffine, affine, kind, walk
from ..ir import dim
from ..ptx import Kernel
from .common import TemplateMismatch
from .gemm import GemmTemplate, _desc_hi, idesc_mma

STATIC_MAX = 48 * 1024 - 256      # static shared memory a kernel may declare
SMEM_LIMIT = 227 * 1024


def meta_only() -> bool:
    """``EMMY_META_ONLY=1``: emit only kernels whose parameters are exactly
    the meta ``arg_order`` (no trailing tensor maps)."""
    return os.environ.get("EMMY_META_ONLY", "") not in ("", "0")


def _strip_mod(e, extent):
    """``(x) % extent`` -> (x, True); anything else -> (e, False)."""
    if kind(e) == "BinaryExpr" and e.op == "%" and kind(e.right) == "Literal" \
            and e.right.value == extent:
        return e.left, True
    return e, False


def _guard_bounds(cond) -> list:
    """The ``x < c`` terms of a guard (``&&`` of comparisons) as (affine x, c)."""
    if kind(cond) == "BinaryExpr" and cond.op in ("&&", "and"):
        return _guard_bounds(cond.left) + _guard_bounds(cond.right)
    if kind(cond) == "BinaryExpr" and cond.op == "<" and kind(cond.right) == "Literal":
        return [(affine(cond.left), int(cond.right.value))]
    raise NotAffine("guard")


def block_indices(k, cta, tile, block_axes) -> dict:
    """Registers holding each block axis's index for CTA ``cta``, as the
    reference decodes the flat thread index when the thread axes fill the CTA
    (``compile.py:2385-2466``): row-major over the block axes, except that a
    grouped rasterisation (``raster_group`` >= 2 over two adjacent axes whose
    grouped one has an extent above 1) numbers ``g`` block rows of the
    grouped axis fastest within each stripe of the other, with a short last
    group when the extent is not a multiple of ``g``."""
    names = [n for n, _ in block_axes]
    ext = dict(block_axes)
    out = {}
    raster = None
    rg, ra = getattr(tile, "raster_group", None), getattr(tile, "raster_axes", None)
    if rg and ra and ra[0] in names and ra[1] in names:
        mi, ni = names.index(ra[0]), names.index(ra[1])
        if ni == mi + 1:
            gi, oi = (mi, ni) if getattr(tile, "raster_orient", None) == "m" else (ni, mi)
            g = min(rg, ext[names[gi]])
            if ext[names[gi]] > 1 and g > 1:
                raster = (gi, oi, g)

    def after(i):
        p = 1
        for n in names[i + 1:]:
            p *= ext[n]
        return p
    for i, n in enumerate(names):
        if raster is not None and i in raster[:2]:
            continue
        r = k.reg("r")
        if ext[n] == 1:
            k(f"mov.u32 {r}, 0;")
        else:
            k(f"div.u32 {r}, {cta}, {after(i)};")
            if i:
                k(f"rem.u32 {r}, {r}, {ext[n]};")
        out[n] = r
    if raster is not None:
        gi, oi, g = raster
        ea, eb = ext[names[gi]], ext[names[oi]]
        mi, ni = min(gi, oi), max(gi, oi)
        sub = k.reg("r")
        k(f"div.u32 {sub}, {cta}, {after(ni)};")
        if mi != 0:
            k(f"rem.u32 {sub}, {sub}, {ea * eb};")
        a, b = k.reg("r"), k.reg("r")
        if ea % g == 0:
            t = k.reg("r")
            k(f"div.u32 {t}, {sub}, {g * eb};")
            k(f"rem.u32 {a}, {sub}, {g};")
            k(f"mad.lo.u32 {a}, {t}, {g}, {a};")
            k(f"rem.u32 {b}, {sub}, {g * eb};")
            k(f"div.u32 {b}, {b}, {g};")
        else:
            grp, rem, rsz = k.reg("r"), k.reg("r"), k.reg("r")
            k(f"div.u32 {grp}, {sub}, {g * eb};")
            k(f"rem.u32 {rem}, {sub}, {g * eb};")
            k(f"mul.lo.u32 {rsz}, {grp}, {g};")
            k(f"sub.u32 {rsz}, {ea}, {rsz};")
            k(f"min.u32 {rsz}, {rsz}, {g};")
            k(f"rem.u32 {a}, {rem}, {rsz};")
            k(f"mad.lo.u32 {a}, {grp}, {g}, {a};")
            k(f"div.u32 {b}, {rem}, {rsz};")
        out[names[gi]], out[names[oi]] = a, b
    return out


class Stager:
    """A CTA's threads staging row-major global operands, 16 bytes at a time,
    into the 128-byte-swizzle K-major layout a tcgen05 shared-memory
    descriptor reads (8-row atoms of 1024 bytes; the 16-byte chunk c of row
    r at chunk c ^ (r % 8)).  A slab is 128 bytes of K per row (32 fp32 or
    64 bf16).  ``fetch`` issues one slab's loads into registers (they stay in
    flight until ``put`` stores them); for fp32 operands ``put`` also writes
    the low tf32 parts lo = x - (x with its 13 low mantissa bits cleared)
    at ``lo_off`` bytes from each chunk (3xTF32)."""

    def __init__(self, k, tid, T, es, tf32):
        self.k, self.tid, self.T, self.es, self.tf32 = k, tid, T, es, tf32
        self.CE = 16 // es               # elements per 16-byte chunk
        self.KB = 128 // es              # k per slab

    def swz(self, row, ch):
        """Byte offset of 16-byte chunk ``ch`` of row ``row``."""
        k = self.k
        o = k.reg("r")
        k(f"and.b32 {o}, {row}, 7;")
        x = k.reg("r")
        k(f"xor.b32 {x}, {ch}, {o};")
        k(f"shl.b32 {x}, {x}, 4;")
        k(f"shl.b32 {o}, {o}, 7;")
        k(f"add.u32 {x}, {x}, {o};")
        a = k.reg("r")
        k(f"shr.u32 {a}, {row}, 3;")
        k(f"mad.lo.u32 {x}, {a}, 1024, {x};")
        return x

    def store_chunk(self, dst, off, vals, lo_off):
        k = self.k
        a = k.reg("r")
        k(f"add.u32 {a}, {dst}, {off};")
        k(f"st.shared.v4.b32 [{a}], {{{', '.join(vals)}}};")
        if self.tf32:
            lo = []
            for v in vals:
                m_ = k.reg("r")
                k(f"and.b32 {m_}, {v}, -8192;")
                l_ = k.reg("r")
                k(f"sub.rn.f32 {l_}, {v}, {m_};")
                lo.append(l_)
            k(f"st.shared.v4.b32 [{a}+{lo_off}], {{{', '.join(lo)}}};")

    def load_elem(self, ptr_base, eidx, ok, dst):
        """dst = element eidx of a global operand if ok, else 0."""
        k, es = self.k, self.es
        k(f"mov.b32 {dst}, 0;")
        a = k.reg("rd")
        k(f"mul.wide.u32 {a}, {eidx}, {es};")
        k(f"add.s64 {a}, {a}, {ptr_base};")
        if es == 4:
            k(f"@{ok} ld.global.nc.b32 {dst}, [{a}];")
        else:
            h = k.reg("h")
            k(f"mov.b16 {h}, 0;")
            k(f"@{ok} ld.global.nc.b16 {h}, [{a}];")
            k(f"cvt.u32.u16 {dst}, {h};")

    def pack16(self, lo16, hi16):
        k = self.k
        r_ = k.reg("r")
        k(f"shl.b32 {r_}, {hi16}, 16;")
        k(f"or.b32 {r_}, {r_}, {lo16};")
        return r_

    def fetch(self, form, kb, base, count, bound, ptr, ld, kend, vec=False, into=None):
        """This thread's chunks of one slab of ``count`` operand rows starting
        at row ``base`` (rows >= ``bound`` and k >= ``kend`` read as 0), k
        from ``kb``.  ``form`` "K": the operand is stored [row][k] (row
        stride ``ld`` elements; ``vec``: a chunk is all in or all out of
        range and 16-byte aligned, one vector load); "T": it is stored
        [k][row] (stride ``ld``): CE loads of one column per chunk,
        coalesced across the threads.  ``into``: the registers of an
        earlier fetch to reuse (a loop-carried register set)."""
        k, T, CE = self.k, self.T, self.CE
        out = []
        slots = iter(into or [])
        for c in range(-(-count * 8 // T)):
            prev = next(slots, None)
            idx = k.reg("r")
            k(f"add.u32 {idx}, {self.tid}, {c * T};")
            live = prev[2] if prev else k.reg("p")
            k(f"setp.lt.u32 {live}, {idx}, {count * 8};")
            row = prev[0] if prev else k.reg("r")
            ch = prev[1] if prev else k.reg("r")
            if form == "K":
                k(f"shr.u32 {row}, {idx}, 3;")
                k(f"and.b32 {ch}, {idx}, 7;")
            else:
                k(f"rem.u32 {row}, {idx}, {count};")
                k(f"div.u32 {ch}, {idx}, {count};")
            g = k.reg("r")
            k(f"add.u32 {g}, {base}, {row};")
            k(f"setp.lt.and.u32 {live}, {g}, {bound}, {live};")
            kk = k.reg("r")
            k(f"mad.lo.u32 {kk}, {ch}, {CE}, {kb};")
            w = prev[3] if prev else k.regs("r", 4)
            for r_ in w:
                k(f"mov.b32 {r_}, 0;")
            if form == "K" and vec:
                ok = k.reg("p")
                k(f"setp.lt.and.u32 {ok}, {kk}, {kend}, {live};")
                ei = k.reg("r")
                k(f"mad.lo.u32 {ei}, {g}, {ld}, {kk};")
                a = k.reg("rd")
                k(f"mul.wide.u32 {a}, {ei}, {self.es};")
                k(f"add.s64 {a}, {a}, {ptr};")
                k(f"@{ok} ld.global.nc.v4.b32 {{{', '.join(w)}}}, [{a}];")
            else:
                elems = k.regs("r", CE)
                for e in range(CE):
                    ke = k.reg("r")
                    k(f"add.u32 {ke}, {kk}, {e};")
                    ok = k.reg("p")
                    k(f"setp.lt.and.u32 {ok}, {ke}, {kend}, {live};")
                    ei = k.reg("r")
                    if form == "K":
                        k(f"mad.lo.u32 {ei}, {g}, {ld}, {ke};")
                    else:
                        k(f"mad.lo.u32 {ei}, {ke}, {ld}, {g};")
                    self.load_elem(ptr, ei, ok, elems[e])
                words = elems if self.es == 4 else [self.pack16(elems[2 * x], elems[2 * x + 1])
                                                    for x in range(4)]
                for r_, x in zip(w, words):
                    k(f"mov.b32 {r_}, {x};")
            out.append((row, ch, live, w))
        return out

    def fetch_mn(self, kb, n0, cols, bound, ptr, ld, kend, into=None):
        """This thread's 16-byte chunks of one slab of a [k][n] operand kept
        MN-major: a chunk is ``CE`` consecutive n of one k row, one vector
        load, coalesced across the threads; in shared memory, blocks of 128
        bytes of n (64 bf16 or 32 fp32 columns) x ``KB`` k rows (block b at
        b * KB * 128, k row r at r * 128 in it) -- the 128-byte-swizzle
        MN-major layouts: bf16 with 16-byte atoms (chunk cc of row r at
        chunk cc ^ (r % 8)), fp32 (tf32) with 32-byte atoms (the 32-byte
        atom cc / 2 of row r at atom (cc / 2) ^ (r % 4), its half cc % 2
        kept).  ``bound`` (the matrix width) is a multiple of ``CE``, so a
        chunk is all in or all out.  Returns chunks as (byte offset, None,
        live, words)."""
        k, T = self.k, self.T
        per_row = cols // self.CE
        out = []
        slots = iter(into or [])
        for c in range(-(-self.KB * per_row // T)):
            prev = next(slots, None)
            idx = k.reg("r")
            k(f"add.u32 {idx}, {self.tid}, {c * T};")
            live = prev[2] if prev else k.reg("p")
            k(f"setp.lt.u32 {live}, {idx}, {self.KB * per_row};")
            kr, nc = k.reg("r"), k.reg("r")
            k(f"div.u32 {kr}, {idx}, {per_row};")
            k(f"rem.u32 {nc}, {idx}, {per_row};")
            off = prev[0] if prev else k.reg("r")
            blk = k.reg("r")
            k(f"shr.u32 {blk}, {nc}, 3;")              # 64-column block
            cc = k.reg("r")
            k(f"and.b32 {cc}, {nc}, 7;")
            k(f"mul.lo.u32 {off}, {blk}, {self.KB * 128};")
            if self.es == 2:
                x = self.swz(kr, cc)
            else:
                x = k.reg("r")                      # 32-byte atoms, 4-row pattern
                r4 = k.reg("r")
                k(f"and.b32 {r4}, {kr}, 3;")
                k(f"shr.u32 {x}, {cc}, 1;")
                k(f"xor.b32 {x}, {x}, {r4};")
                k(f"shl.b32 {x}, {x}, 5;")
                h = k.reg("r")
                k(f"and.b32 {h}, {cc}, 1;")
                k(f"mad.lo.u32 {x}, {h}, 16, {x};")
                k(f"mad.lo.u32 {x}, {kr}, 128, {x};")
            k(f"add.u32 {off}, {off}, {x};")
            gk = k.reg("r")
            k(f"add.u32 {gk}, {kb}, {kr};")
            gn = k.reg("r")
            k(f"mad.lo.u32 {gn}, {nc}, {self.CE}, {n0};")
            ok = k.reg("p")
            k(f"setp.lt.and.u32 {ok}, {gk}, {kend}, {live};")
            k(f"setp.lt.and.u32 {ok}, {gn}, {bound}, {ok};")
            w = prev[3] if prev else k.regs("r", 4)
            for r_ in w:
                k(f"mov.b32 {r_}, 0;")
            ei = k.reg("r")
            k(f"mad.lo.u32 {ei}, {gk}, {ld}, {gn};")
            a = k.reg("rd")
            k(f"mul.wide.u32 {a}, {ei}, {self.es};")
            k(f"add.s64 {a}, {a}, {ptr};")
            k(f"@{ok} ld.global.nc.v4.b32 {{{', '.join(w)}}}, [{a}];")
            out.append((off, None, live, w))
        return out

    def put(self, chunks, dst, lo_off):
        """Store fetched chunks at buffer ``dst`` (a register)."""
        k = self.k
        for row, ch, live, w in chunks:
            sk = k.label("NO_CHUNK")
            k(f"@!{live} bra {sk};")
            self.store_chunk(dst, row if ch is None else self.swz(row, ch), w, lo_off)
            k.mark(sk)


class GemmSmallTemplate:
    name = "gemm"
    # a CTA whose threads own fewer multiply-adds than this each runs
    # faster through the generic lowering (FFMA): the tensor-memory
    # allocation, barriers and staging outweigh the products.  Measured on
    # Emmy's own matmul IRs (per-thread multiply-adds: this template /
    # generic, us): m02 16: 12.3 / 6.2, mm256 48: 31.2 / 10.8, mm64a 64:
    # 8.7 / 6.7, mm_rect2 64: 8.6 / 6.7, mm128 1536: 10.8 / 8.7, m01 and
    # mm512 2048: 21.0 / 98.8
    MIN_MACS_PER_THREAD = 2048
    # by operand mode: CTAs of two or more warps issue the MMAs from a warp
    # of their own (the others only stage), else thread 0 stages and issues.
    # Measured on one B200 (same process, alternating, outputs checked):
    # 3xTF32, whose slab holds three products a k step, m01 21.0-21.8 ->
    # 18.8 us and the meta-only BASELINE fp32 matmul 7.76 -> 7.48 ms; bf16,
    # bound by staging, 4.97 -> 5.17 ms with one warp fewer staging
    DEDICATED_ISSUER = {"tf32x3": True, "bf16": False}
    # bf16 B staged MN-major (16-byte loads along N, no transposition).
    # Measured on one B200 (same process, alternating, outputs checked): the
    # meta-only BASELINE bf16 matmul 4.96-4.98 -> 2.89-2.90 ms (221 -> 380
    # TFLOP/s)
    BF16_B_MN = True
    # bf16 operands copied global -> shared by cp.async (16-byte chunks,
    # zero-filled past the matrix) into a ring of 3-4 buffers, up to two
    # slabs in flight beyond the one being multiplied, no register staging.
    # Measured the same way: the meta-only BASELINE bf16 matmul 2.885-2.888
    # -> 2.042-2.044 ms (381 -> 538 TFLOP/s)
    ASYNC_BF16 = True
    # fp32 B staged MN-major too (the tf32 MN-major layout: 32-byte atoms).
    # Measured the same way: the meta-only BASELINE fp32 matmul 7.46 ->
    # 6.16 ms (147 -> 178 TFLOP/s); m01 18.9 us either way (issue-bound)
    TF32_B_MN = True

    # ------------------------------------------------------------------ match
    @classmethod
    def match(cls, ctx) -> "GemmSmallTemplate":
        tile = ctx.tile
        if tile is None:
            raise TemplateMismatch("no single top-level Tile")
        if getattr(tile, "aux_threads", 0):
            raise TemplateMismatch("auxiliary-thread tile")
        axes = ctx.tile_axes()
        names = [a for a, _ in axes]
        if names[-4:] != ["a0_b", "a1_b", "a0_u", "a1_u"] or len(names) not in (4, 5):
            raise TemplateMismatch("not a matmul tile (..., a0_b, a1_b, a0_u, a1_u)")
        ext = dict(axes)
        ks_axis = names[0] if len(names) == 5 else None
        T = ext["a0_u"] * ext["a1_u"]
        bt = getattr(tile, "block_threads", None)
        if ctx.block != (T, 1, 1) or (bt not in (None, T)) or T % 32 or T > 1024:
            raise TemplateMismatch("CTA is not the a0_u x a1_u thread block")
        nblk = ext["a0_b"] * ext["a1_b"] * (ext[ks_axis] if ks_axis else 1)
        if ctx.grid[0] * ctx.grid[1] * ctx.grid[2] != nblk:
            raise TemplateMismatch("grid is not one CTA per (k chunk, tile)")
        body = list(walk(tile.body))
        smems = {s.name for s in body if kind(s) == "Smem"}
        copies = [s for s in body if kind(s) == "CpAsyncCopy"]
        inits = {s.name for s in body if kind(s) == "Init"}
        if len(smems) != 2 or not copies or not inits:
            raise TemplateMismatch("matmul statements missing")
        if any(float(s.identity) != 0.0 for s in body if kind(s) == "Init"):
            raise TemplateMismatch("accumulator not zero-initialised")
        src_of = {}
        for c in copies:
            if src_of.setdefault(c.smem, c.src) != c.src:
                raise TemplateMismatch("smem filled from two buffers")
        loops = [s for s in body if kind(s) == "Loop"]
        if len(loops) != 1:
            raise TemplateMismatch("expected one inner k loop")
        role, defs, pairs = {}, {}, set()
        for s in loops[0].body:
            k_ = kind(s)
            if k_ == "Load":
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
            elif k_ == "Assign":
                if s.op.name != "multiply" or len(s.args) != 2:
                    raise TemplateMismatch(f"inner op {s.op.name}")
                a, b = (defs.get(x) for x in s.args)
                if not (a and b and a[0] == b[0] == "load" and a[1] != b[1]):
                    raise TemplateMismatch("multiply of non-smem operands")
                defs[s.name] = ("mul", frozenset((a[1], b[1])))
            elif k_ == "Accum":
                if s.name not in inits or s.op.name != "add" or s.base:
                    raise TemplateMismatch("accumulate shape")
                v = defs.get(s.value)
                if not v or v[0] != "mul":
                    raise TemplateMismatch("accumulate of a non-product")
                pairs.add(v[1])
            else:
                raise TemplateMismatch(f"{k_} in the inner k loop")
        if pairs != {frozenset(smems)}:
            raise TemplateMismatch("products do not pair the two smem tiles")
        inv = {v: s for s, v in role.items()}
        if set(inv) != {"A", "B"}:
            raise TemplateMismatch("operand roles")
        A, B = src_of.get(inv["A"]), src_of.get(inv["B"])
        bufs = ctx.bufs
        # the stores: (row, col) of each value, possibly as (x % extent)
        # under a Cond(x < extent) guard
        writes = []

        def collect(stmts, guards):
            for s in stmts:
                k_ = kind(s)
                if k_ == "Write":
                    writes.append((s, guards))
                elif k_ == "Cond":
                    if s.else_body:
                        raise TemplateMismatch("store under if/else")
                    try:
                        g = _guard_bounds(s.cond)
                    except NotAffine as e:
                        raise TemplateMismatch(f"store guard: {e}")
                    collect(s.body, guards + g)
                elif k_ in ("Loop", "StridedLoop"):
                    if any(kind(x) == "Write" for x in walk(s.body)):
                        raise TemplateMismatch("store inside a loop")
        collect(tile.body, [])
        if not writes:
            raise TemplateMismatch("no stores")
        outs = {w.output for w, _ in writes}
        if len(outs) != 1:
            raise TemplateMismatch("multiple outputs")
        C = outs.pop()
        if A is None or B is None or any(len(bufs.shapes.get(x, ())) != 2 for x in (A, B, C)):
            raise TemplateMismatch("operand ranks")
        M, K = bufs.shapes[A]
        K2, N = bufs.shapes[B]
        if K2 != K or tuple(bufs.shapes[C]) != (M, N) or bufs.dtypes.get(C) != "f32":
            raise TemplateMismatch("operand shapes")
        atomic = {w.atomic for w, _ in writes}
        if len(atomic) != 1:
            raise TemplateMismatch("mixed plain and atomic stores")
        atomic = atomic.pop()
        # atomic stores add the CTA's partial product to C, as the IR's own
        # red.global.add does, whatever C held before (the runner zeroes it)
        if not atomic and ks_axis is not None and ext[ks_axis] > 1:
            raise TemplateMismatch("split K with plain stores")
        BM = BN = mu = nu = None
        cells = set()
        for w, guards in writes:
            if len(w.index) != 2:
                raise TemplateMismatch("store rank")
            try:
                re_, rmod = _strip_mod(w.index[0], M)
                ce_, cmod = _strip_mod(w.index[1], N)
                r, c = affine(re_), affine(ce_)
            except NotAffine as e:
                raise TemplateMismatch(f"store index: {e}")
            # a wrapped index is only the identity where a guard bounds it
            for x, wrapped, bound in ((r, rmod, M), (c, cmod, N)):
                if wrapped and not any(gx == x and gc <= bound for gx, gc in guards):
                    raise TemplateMismatch("wrapped store index without its guard")
            for gx, gc in guards:
                if gx != r and gx != c:
                    raise TemplateMismatch("guard on something else than the store index")
            if r.vars() - {"a0_b", "a0_u"} or c.vars() - {"a1_b", "a1_u"}:
                raise TemplateMismatch("store index variables")
            bm, m_, bn, n_ = r.coef("a0_b"), r.coef("a0_u"), c.coef("a1_b"), c.coef("a1_u")
            if BM is None:
                BM, mu, BN, nu = bm, m_, bn, n_
            if (bm, m_, bn, n_) != (BM, mu, BN, nu):
                raise TemplateMismatch("stores disagree on the tile")
            for j in range(len(w.values)):
                cells.add((r.const, c.const + j))
        if not mu or not nu or BM != ext["a0_u"] * mu or BN != ext["a1_u"] * nu:
            raise TemplateMismatch("micro-tiles do not tile the CTA tile")
        if cells != {(i, j) for i in range(mu) for j in range(nu)}:
            raise TemplateMismatch("stores do not cover each micro-tile once")
        # rows / columns past the matrix must be guarded, tiles must reach it
        if ext["a0_b"] * BM < M or ext["a1_b"] * BN < N:
            raise TemplateMismatch("tiles do not cover the output")
        for w, guards in writes:
            r = affine(_strip_mod(w.index[0], M)[0])
            c = affine(_strip_mod(w.index[1], N)[0])
            if ext["a0_b"] * BM > M and not any(gx == r for gx, _ in guards):
                raise TemplateMismatch("rows past M stored unguarded")
            if ext["a1_b"] * BN > N and not any(gx == c for gx, _ in guards):
                raise TemplateMismatch("columns past N stored unguarded")
        # the CTA's K range: the k-slab loop's extent; with split K the
        # leading axis numbers the chunks
        kl = [s for s in body if kind(s) == "StridedLoop" and
              any(kind(x) == "Loop" for x in walk(s.body))]
        if len(kl) != 1:
            raise TemplateMismatch("expected one k-slab loop")
        KC = dim(kl[0].axis.extent)
        nks = ext[ks_axis] if ks_axis else 1
        if KC * nks != K:
            raise TemplateMismatch("k chunks do not cover K")
        dts = {bufs.dtypes[A], bufs.dtypes[B]}
        if dts == {"f32"}:
            mode = "tf32x3"
        elif dts == {"bf16"}:
            mode = "bf16"
        else:
            raise TemplateMismatch(f"operand dtypes {dts}")
        warps = T // 32
        if BM > 128 or BM > 32 * min(4, warps) or BN > 256:
            raise TemplateMismatch(f"tile {BM}x{BN} too large for {T} threads")
        if BM * BN * KC < cls.MIN_MACS_PER_THREAD * T:
            raise TemplateMismatch(f"{BM}x{BN}x{KC} per CTA is {BM * BN * KC // T} multiply-adds "
                                   f"a thread: below {cls.MIN_MACS_PER_THREAD}, the generic "
                                   f"lowering is faster")
        self = cls()
        self.ctx, self.A, self.B, self.C = ctx, A, B, C
        self.M, self.N, self.K, self.KC = M, N, K, KC
        self.BM, self.BN, self.T = BM, BN, T
        self.nb0, self.nb1, self.nks = ext["a0_b"], ext["a1_b"], nks
        self.ks_axis = ks_axis
        self.block_axes = axes[:-2]
        self.mode, self.atomic = mode, atomic
        self.es = 4 if mode == "tf32x3" else 2
        self.CE = 16 // self.es                 # elements per 16-byte chunk
        self.KB = 128 // self.es                # k per 128-byte swizzle row (one slab)
        self.BNp = -(-BN // 16) * 16
        # bf16 B kept MN-major (as stored: 16-byte loads along N, no
        # transposition) when the tile is whole 64-column blocks and N a
        # multiple of 8; otherwise transposed into K-major chunks
        self.b_mn = ((cls.BF16_B_MN and mode == "bf16" and self.BNp % 64 == 0 and N % 8 == 0) or
                     (cls.TF32_B_MN and mode == "tf32x3" and self.BNp % 32 == 0 and N % 4 == 0))
        half = 2 if mode == "tf32x3" else 1     # raw + low parts
        # per slab buffer: A (the tile's rows, in whole 8-row atoms) | A_lo |
        # B (BNp rows) | B_lo, 128 bytes a row.  The MMA's A descriptor spans
        # 128 rows (16 KiB) from A's base: rows past the tile read the bytes
        # after it (garbage that only reaches accumulator rows never
        # stored), so the allocation reaches 16 KiB past the last A base
        self.sa = -(-BM // 8) * 1024
        self.sb = self.BNp * 128
        self.buf = (self.sa + self.sb) * half

        def need(nbuf):
            span = (nbuf - 1) * self.buf + (self.sa if half == 2 else 0) + 128 * 128
            return max(nbuf * self.buf, span) + 1024 + 64
        avail = min(ctx.smem_bytes, SMEM_LIMIT)
        # static shared memory adds to the launch's dynamic bytes: a launcher
        # raises the per-CTA limit above 48 KiB only for dynamic sizes above it
        cap = SMEM_LIMIT if avail > 48 * 1024 else 48 * 1024
        # bf16 with both operands in 16-byte chunks (A rows along K, B MN-major)
        # copies global -> shared with cp.async, so a slab needs no registers
        # and up to three slabs are in flight (four buffers)
        self.async_ = bool(cls.ASYNC_BF16 and mode == "bf16" and self.b_mn
                           and K % 8 == 0 and KC % 8 == 0)
        if self.async_:
            # the ring needs three buffers or more (a buffer is refilled one
            # slab after its MMAs are issued), all in dynamic shared memory
            fit = [n for n in (4, 3) if avail >= need(n)]
            self.async_ = bool(fit)
            if fit:
                self.nbuf, self.dynamic = fit[0], True
        for nbuf in (() if self.async_ else (2, 1)):
            if avail >= need(nbuf):
                self.nbuf, self.dynamic = nbuf, True
                break
            if need(nbuf) <= STATIC_MAX and need(nbuf) + avail <= cap:
                self.nbuf, self.dynamic = nbuf, False
                break
        else:
            if not self.async_:
                raise TemplateMismatch("shared memory for one slab")
        self.smem_need = need(self.nbuf)
        return self

    # ------------------------------------------------------------------- emit
    def emit(self) -> str:
        ctx = self.ctx
        T, BM, BN, BNp, KB, CE, es = self.T, self.BM, self.BN, self.BNp, self.KB, self.CE, self.es
        M, N, K, KC = self.M, self.N, self.K, self.KC
        tf32 = self.mode == "tf32x3"
        KMMA = 32 // es                         # k per tcgen05.mma (32 bytes)
        k = Kernel(ctx.entry, ctx.params())
        k.maxntid = (T, 1, 1)
        if self.dynamic:
            k.decl(".extern .shared .align 1024 .b8 __emmy_smem[];")
        else:
            k.decl(f".shared .align 1024 .b8 __emmy_smem[{self.smem_need}];")
        k.decl(".global .align 4 .u32 __emmy_status;")
        k.comment(f"emmy-b200 template: tcgen05 gemm, meta-only launch (no tensor maps), "
                  f"{self.mode} M={M} N={N} K={K}, CTA tile {BM}x{BN} over K chunks of {KC}, "
                  f"{T} threads, {self.nbuf} slab buffer(s)")
        abase, bbase, cbase = k.param_ptr(self.A), k.param_ptr(self.B), k.param_ptr(self.C)
        tid = k.special("%tid.x")
        warp = k.reg("r")
        k(f"shr.u32 {warp}, {tid}, 5;")
        lane = k.reg("r")
        k(f"and.b32 {lane}, {tid}, 31;")
        cta = k.special("%ctaid.x")
        blk = block_indices(k, cta, ctx.tile, self.block_axes)
        mb, nb = blk["a0_b"], blk["a1_b"]
        ks = blk.get(self.ks_axis) if self.ks_axis else k.reg("r")
        if not self.ks_axis:
            k(f"mov.u32 {ks}, 0;")
        r0 = k.reg("r")
        k(f"mul.lo.u32 {r0}, {mb}, {BM};")
        n0 = k.reg("r")
        k(f"mul.lo.u32 {n0}, {nb}, {BN};")
        k0 = k.reg("r")
        k(f"mul.lo.u32 {k0}, {ks}, {KC};")
        kend = k.reg("r")
        k(f"add.u32 {kend}, {k0}, {KC};")
        # shared memory: nbuf x [A | A_lo | B | B_lo], then barriers, tmem slot
        raw = k.reg("r")
        k(f"mov.u32 {raw}, __emmy_smem;")
        sm = k.reg("r")
        k(f"add.u32 {sm}, {raw}, 1023;")
        k(f"and.b32 {sm}, {sm}, -1024;")
        bars = k.reg("r")
        k(f"add.u32 {bars}, {sm}, {self.smem_need - 1024 - 64};")
        tslot = k.reg("r")
        k(f"add.u32 {tslot}, {bars}, 48;")
        status = k.reg("rd")
        k(f"mov.u64 {status}, __emmy_status;")
        p0 = k.reg("p")
        k(f"setp.eq.u32 {p0}, {tid}, 0;")
        skip = k.label("SKIP_INIT")
        k(f"@!{p0} bra {skip};")
        # a CTA of two or more warps gives its last warp to the MMA issue:
        # the others stage slabs and arrive on the buffer's STAGED barrier
        # (one arrival a thread), so no staging thread waits for an issue
        dedicated = self.DEDICATED_ISSUER.get(self.mode, False) and T >= 64
        T_st = T - 32 if dedicated else T
        for b in range(self.nbuf):
            k(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * b}], 1;")
            if dedicated:
                k(f"mbarrier.init.shared::cta.b64 [{bars}+{32 + 8 * b}], {T_st};")
        k("fence.mbarrier_init.release.cluster;")
        k.mark(skip)
        pw0 = k.reg("p")
        k(f"setp.eq.u32 {pw0}, {warp}, 0;")
        skip2 = k.label("SKIP_ALLOC")
        ncols = max(32, 1 << (BNp - 1).bit_length())
        k(f"@!{pw0} bra {skip2};")
        k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{tslot}], {ncols};")
        k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
        k.mark(skip2)
        k("tcgen05.fence::before_thread_sync;")
        k("bar.sync 0;")
        k("tcgen05.fence::after_thread_sync;")
        tmem = k.reg("r")
        k(f"ld.shared.u32 {tmem}, [{tslot}];")
        teardown = k.label("TEARDOWN")
        idesc = k.reg("r")
        bmn = self.b_mn
        k(f"mov.u32 {idesc}, {idesc_mma(128, BNp, bmn, tf32)};")
        hi = _desc_hi(16, 1024)
        hiB = (hi if not bmn else _desc_hi(KB * 128, 512, 1) if tf32
               else _desc_hi(KB * 128, 1024))
        ptrue = k.reg("p")
        k(f"setp.eq.u32 {ptrue}, 0, 0;")
        wait = GemmTemplate._wait

        st = Stager(k, tid, T_st, es, tf32)

        vec_a = K % CE == 0 and KC % CE == 0            # a chunk is all in or all out

        def fetch(slab, into=None):
            """This thread's A and B chunks of slab ``slab`` (k from k0 + slab*KB)."""
            kb = k.reg("r")
            k(f"mad.lo.u32 {kb}, {slab}, {KB}, {k0};")
            na = -(-BM * 8 // T_st)              # A chunks a staging thread holds
            a = st.fetch("K", kb, r0, BM, M, abase, K, kend, vec_a, into and into[:na])
            if bmn:
                b = st.fetch_mn(kb, n0, BNp, N, bbase, N, kend, into and into[na:])
            else:
                b = st.fetch("T", kb, n0, BN, N, bbase, N, kend, False, into and into[na:])
            return a + b, na

        def put(fetched, buf):
            """Store a fetch into slab buffer ``buf``: A | A_lo | B | B_lo."""
            chunks, na = fetched
            base = k.reg("r")
            k(f"mad.lo.u32 {base}, {buf}, {self.buf}, {sm};")
            st.put(chunks[:na], base, self.sa)
            bb = k.reg("r")
            k(f"add.u32 {bb}, {base}, {self.sa * (2 if tf32 else 1)};")
            st.put(chunks[na:], bb, self.sb)
            k("fence.proxy.async.shared::cta;")

        def mma(slab, buf, nsteps, issuer=p0):
            """Thread ``issuer``: the MMAs of one staged slab, then a commit."""
            sk = k.label("NO_MMA")
            k(f"@!{issuer} bra {sk};")
            k("tcgen05.fence::after_thread_sync;")
            base = k.reg("r")
            k(f"mad.lo.u32 {base}, {buf}, {self.buf}, {sm};")
            da = GemmTemplate._desc(k, base, hi)
            bb = k.reg("r")
            k(f"add.u32 {bb}, {base}, {self.sa * (2 if tf32 else 1)};")
            db = GemmTemplate._desc(k, bb, hiB)
            bstep = KMMA * 8 if bmn else 2          # a K step: KMMA k rows MN-major, 32 bytes K-major
            if tf32:
                la = k.reg("r")
                k(f"add.u32 {la}, {base}, {self.sa};")
                dla = GemmTemplate._desc(k, la, hi)
                lb = k.reg("r")
                k(f"add.u32 {lb}, {base}, {2 * self.sa + self.sb};")
                dlb = GemmTemplate._desc(k, lb, hiB)
            pacc = k.reg("p")
            k(f"setp.ne.u32 {pacc}, {slab}, 0;")
            first = True
            for st in range(nsteps):
                pairs = [(dla, db), (da, dlb), (da, db)] if tf32 else [(da, db)]
                for x, y in pairs:
                    ax = k.reg("rd")
                    k(f"add.s64 {ax}, {x}, {2 * st};")
                    by = k.reg("rd")
                    k(f"add.s64 {by}, {y}, {bstep * st};")
                    kind_ = "tf32" if tf32 else "f16"
                    k(f"tcgen05.mma.cta_group::1.kind::{kind_} [{tmem}], {ax}, {by}, {idesc}, "
                      f"{pacc if first else ptrue};")
                    first = False
            bar = k.reg("r")
            k(f"mad.lo.u32 {bar}, {buf}, 8, {bars};")
            k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{bar}];")
            k.mark(sk)

        def wait_slab(slab):
            """Wait for the MMAs of slab ``slab`` (its buffer's barrier,
            completion number slab // nbuf)."""
            b = k.reg("r")
            k(f"rem.u32 {b}, {slab}, {self.nbuf};")
            bar = k.reg("r")
            k(f"mad.lo.u32 {bar}, {b}, 8, {bars};")
            ph = k.reg("r")
            k(f"div.u32 {ph}, {slab}, {self.nbuf};")
            k(f"and.b32 {ph}, {ph}, 1;")
            wait(k, bar, ph, status, 2, teardown)

        nslab = -(-KC // KB)
        s = k.reg("r")
        bufr = k.reg("r")

        def copy_async(slab, buf):
            """cp.async of slab ``slab`` (a register) into buffer ``buf`` (a
            register): this thread's 16-byte chunks of A (rows along K) and of
            B (MN-major), zero-filled outside the matrix and the K range."""
            base = k.reg("r")
            k(f"mad.lo.u32 {base}, {buf}, {self.buf}, {sm};")
            kb = k.reg("r")
            k(f"mad.lo.u32 {kb}, {slab}, {KB}, {k0};")

            def chunk(live, ok, dst, gidx, ptr):
                src = k.reg("rd")
                k(f"mul.wide.u32 {src}, {gidx}, {es};")
                k(f"add.s64 {src}, {src}, {ptr};")
                k(f"selp.b64 {src}, {src}, {ptr}, {ok};")      # no read when zero-filled
                sz = k.reg("r")
                k(f"selp.u32 {sz}, 16, 0, {ok};")
                k(f"@{live} cp.async.cg.shared.global [{dst}], [{src}], 16, {sz};")
            for c in range(-(-BM * 8 // T)):
                idx = k.reg("r")
                k(f"add.u32 {idx}, {tid}, {c * T};")
                live = k.reg("p")
                k(f"setp.lt.u32 {live}, {idx}, {BM * 8};")
                row, ch = k.reg("r"), k.reg("r")
                k(f"shr.u32 {row}, {idx}, 3;")
                k(f"and.b32 {ch}, {idx}, 7;")
                g = k.reg("r")
                k(f"add.u32 {g}, {r0}, {row};")
                kk = k.reg("r")
                k(f"mad.lo.u32 {kk}, {ch}, {CE}, {kb};")
                ok = k.reg("p")
                k(f"setp.lt.and.u32 {ok}, {g}, {M}, {live};")
                k(f"setp.lt.and.u32 {ok}, {kk}, {kend}, {ok};")
                dst = k.reg("r")
                k(f"add.u32 {dst}, {base}, {st.swz(row, ch)};")
                gi = k.reg("r")
                k(f"mad.lo.u32 {gi}, {g}, {K}, {kk};")
                chunk(live, ok, dst, gi, abase)
            per_row = BNp // CE
            for c in range(-(-KB * per_row // T)):
                idx = k.reg("r")
                k(f"add.u32 {idx}, {tid}, {c * T};")
                live = k.reg("p")
                k(f"setp.lt.u32 {live}, {idx}, {KB * per_row};")
                kr, nc = k.reg("r"), k.reg("r")
                k(f"div.u32 {kr}, {idx}, {per_row};")
                k(f"rem.u32 {nc}, {idx}, {per_row};")
                blk, cc = k.reg("r"), k.reg("r")
                k(f"shr.u32 {blk}, {nc}, 3;")
                k(f"and.b32 {cc}, {nc}, 7;")
                dst = k.reg("r")
                k(f"mad.lo.u32 {dst}, {blk}, {KB * 128}, {base};")
                k(f"add.u32 {dst}, {dst}, {st.swz(kr, cc)};")
                k(f"add.u32 {dst}, {dst}, {self.sa};")
                gk, gn = k.reg("r"), k.reg("r")
                k(f"add.u32 {gk}, {kb}, {kr};")
                k(f"mad.lo.u32 {gn}, {nc}, {CE}, {n0};")
                ok = k.reg("p")
                k(f"setp.lt.and.u32 {ok}, {gk}, {kend}, {live};")
                k(f"setp.lt.and.u32 {ok}, {gn}, {N}, {ok};")
                gi = k.reg("r")
                k(f"mad.lo.u32 {gi}, {gk}, {N}, {gn};")
                chunk(live, ok, dst, gi, bbase)

        if self.async_:
            # one commit group per prologue slab and one per iteration (empty
            # when nothing is refilled): slab t >= D is copied in iteration
            # t - D + 1, so when iteration s waits for slab s, at most D - 2
            # newer groups may still be pending (D - 1 for the prologue's
            # slabs: waiting for D - 2 is stricter, never wrong)
            D = self.nbuf
            for i in range(D):
                if i < nslab:
                    ri = k.reg("r")
                    k(f"mov.u32 {ri}, {i};")
                    copy_async(ri, ri)
                k("cp.async.commit_group;")
            k(f"mov.u32 {s}, 0;")
            top = k.label("SLAB")
            k.mark(top)
            k(f"cp.async.wait_group {D - 2};")
            k("fence.proxy.async.shared::cta;")
            k("bar.sync 0;")
            k(f"rem.u32 {bufr}, {s}, {D};")
            mma(s, bufr, KB // KMMA)
            # refill the buffer of slab s-1 (its MMAs were issued a slab ago)
            # with slab s-1+D
            skr = k.label("NO_REFILL")
            pr = k.reg("p")
            k(f"setp.eq.u32 {pr}, {s}, 0;")
            k(f"@{pr} bra {skr};")
            prv = k.reg("r")
            k(f"sub.u32 {prv}, {s}, 1;")
            nx = k.reg("r")
            k(f"add.u32 {nx}, {prv}, {D};")
            pn2 = k.reg("p")
            k(f"setp.ge.u32 {pn2}, {nx}, {nslab};")
            k(f"@{pn2} bra {skr};")
            wait_slab(prv)
            pb = k.reg("r")
            k(f"rem.u32 {pb}, {prv}, {D};")
            copy_async(nx, pb)
            k.mark(skr)
            k("cp.async.commit_group;")
            k(f"add.u32 {s}, {s}, 1;")
            pl = k.reg("p")
            k(f"setp.lt.u32 {pl}, {s}, {nslab};")
            k(f"@{pl} bra {top};")
            last = k.reg("r")
            k(f"mov.u32 {last}, {nslab - 1};")
            wait_slab(last)                       # MMAs complete in order: all done
            k("cp.async.wait_group 0;")
        elif dedicated:
            after = k.label("STAGED_ALL")
            pmw = k.reg("p")                      # the MMA warp
            k(f"setp.eq.u32 {pmw}, {warp}, {T // 32 - 1};")
            mloop = k.label("MMA_WARP")
            k(f"@{pmw} bra {mloop};")
            # staging warps: slab s into buffer s % nbuf once the MMAs that
            # read the buffer's previous slab are done, then one arrival a
            # thread on the buffer's STAGED barrier; the next slab's loads
            # are in flight in registers meanwhile
            k(f"mov.u32 {s}, 0;")
            chunks = fetch(s)
            top = k.label("SLAB")
            k.mark(top)
            k(f"rem.u32 {bufr}, {s}, {self.nbuf};")
            pw = k.reg("p")
            k(f"setp.ge.u32 {pw}, {s}, {self.nbuf};")
            skw = k.label("NO_WAIT")
            k(f"@!{pw} bra {skw};")
            prev = k.reg("r")
            k(f"sub.u32 {prev}, {s}, {self.nbuf};")
            wait_slab(prev)                       # the buffer's previous MMAs are done
            k.mark(skw)
            put(chunks, bufr)                     # ends with the async-proxy fence
            sbar = k.reg("r")
            k(f"mad.lo.u32 {sbar}, {bufr}, 8, {bars};")
            k(f"mbarrier.arrive.shared::cta.b64 _, [{sbar}+32];")
            nxt = k.reg("r")
            k(f"add.u32 {nxt}, {s}, 1;")
            pn = k.reg("p")
            k(f"setp.lt.u32 {pn}, {nxt}, {nslab};")
            skf = k.label("NO_FETCH")
            k(f"@!{pn} bra {skf};")
            fetch(nxt, chunks[0])
            k.mark(skf)
            k(f"mov.u32 {s}, {nxt};")
            k(f"@{pn} bra {top};")
            k(f"bra {after};")
            # the MMA warp's lane 0: slab s once its buffer is staged
            k.mark(mloop)
            pl0 = k.reg("p")
            k(f"setp.eq.u32 {pl0}, {lane}, 0;")
            k(f"@!{pl0} bra {after};")
            k(f"mov.u32 {s}, 0;")
            mtop = k.label("MMA_SLAB")
            k.mark(mtop)
            k(f"rem.u32 {bufr}, {s}, {self.nbuf};")
            sbar2 = k.reg("r")
            k(f"mad.lo.u32 {sbar2}, {bufr}, 8, {bars};")
            k(f"add.u32 {sbar2}, {sbar2}, 32;")
            sph = k.reg("r")
            k(f"div.u32 {sph}, {s}, {self.nbuf};")
            k(f"and.b32 {sph}, {sph}, 1;")
            wait(k, sbar2, sph, status, 2, teardown)
            mma(s, bufr, KB // KMMA, issuer=ptrue)
            k(f"add.u32 {s}, {s}, 1;")
            pm = k.reg("p")
            k(f"setp.lt.u32 {pm}, {s}, {nslab};")
            k(f"@{pm} bra {mtop};")
            k.mark(after)
            last = k.reg("r")
            k(f"mov.u32 {last}, {nslab - 1};")
            wait_slab(last)                       # MMAs complete in order: all done
            k("bar.warp.sync 0xffffffff;")
        else:
            k(f"mov.u32 {s}, 0;")
            chunks = fetch(s)
            top = k.label("SLAB")
            k.mark(top)
            k(f"rem.u32 {bufr}, {s}, {self.nbuf};")
            pw = k.reg("p")
            k(f"setp.ge.u32 {pw}, {s}, {self.nbuf};")
            skw = k.label("NO_WAIT")
            k(f"@!{pw} bra {skw};")
            prev = k.reg("r")
            k(f"sub.u32 {prev}, {s}, {self.nbuf};")
            wait_slab(prev)                       # the buffer's previous MMAs are done
            k.mark(skw)
            put(chunks, bufr)
            k("bar.sync 0;")
            nxt = k.reg("r")
            k(f"add.u32 {nxt}, {s}, 1;")
            pn = k.reg("p")
            k(f"setp.lt.u32 {pn}, {nxt}, {nslab};")
            skf = k.label("NO_FETCH")
            k(f"@!{pn} bra {skf};")
            fetch(nxt, chunks[0])                 # in flight while the MMAs run
            k.mark(skf)
            mma(s, bufr, KB // KMMA)
            k(f"mov.u32 {s}, {nxt};")
            k(f"@{pn} bra {top};")
            last = k.reg("r")
            k(f"mov.u32 {last}, {nslab - 1};")
            wait_slab(last)                       # MMAs complete in order: all done
        k("tcgen05.fence::after_thread_sync;")
        # ---------------- epilogue ----------------
        warps = T // 32
        groups = max(1, warps // 4)
        q = k.reg("r")
        k(f"and.b32 {q}, {warp}, 3;")
        g_ = k.reg("r")
        k(f"shr.u32 {g_}, {warp}, 2;")
        skip_ep = k.label("NO_ROWS")
        pq = k.reg("p")
        k(f"setp.ge.u32 {pq}, {q}, {-(-BM // 32)};")       # no tile rows in this quarter
        k(f"@{pq} bra {skip_ep};")
        lrow = k.reg("r")
        k(f"mad.lo.u32 {lrow}, {q}, 32, {lane};")
        grow = k.reg("r")
        k(f"add.u32 {grow}, {r0}, {lrow};")
        rok = k.reg("p")
        k(f"setp.lt.u32 {rok}, {grow}, {M};")
        rok2 = k.reg("p")
        k(f"setp.lt.and.u32 {rok2}, {lrow}, {BM}, {rok};")
        crow = k.reg("rd")
        k(f"mul.wide.u32 {crow}, {grow}, {N * 4};")
        k(f"add.s64 {crow}, {crow}, {cbase};")
        taddr = k.reg("r")
        k(f"shl.b32 {taddr}, {q}, 21;")
        k(f"add.u32 {taddr}, {taddr}, {tmem};")
        chunks = list(range(0, BNp, 8))
        for gi in range(groups):
            mine = [c for i, c in enumerate(chunks) if i % groups == gi]
            if not mine:
                continue
            skg = k.label("NOT_MY_COLS")
            pg = k.reg("p")
            k(f"setp.ne.u32 {pg}, {g_}, {gi};")
            if groups > 1:
                k(f"@{pg} bra {skg};")
            for c in mine:
                regs = k.regs("r", 8)
                k(f"tcgen05.ld.sync.aligned.32x32b.x8.b32 {{{', '.join(regs)}}}, [{taddr}+{c}];")
                k("tcgen05.wait::ld.sync.aligned;")
                for e in range(8):
                    if c + e >= BN:
                        break
                    gc = k.reg("r")
                    k(f"add.u32 {gc}, {n0}, {c + e};")
                    ok = k.reg("p")
                    k(f"setp.lt.and.u32 {ok}, {gc}, {N}, {rok2};")
                    a = k.reg("rd")
                    k(f"mul.wide.u32 {a}, {gc}, 4;")
                    k(f"add.s64 {a}, {a}, {crow};")
                    op = "red.global.add.f32" if self.atomic else "st.global.f32"
                    k(f"@{ok} {op} [{a}], {regs[e]};")
            k.mark(skg)
        k.mark(skip_ep)
        # ---------------- teardown ----------------
        k.mark(teardown)
        k("tcgen05.fence::before_thread_sync;")
        k("barrier.sync 0;")
        end = k.label("END")
        k(f"@!{pw0} bra {end};")
        k("bar.warp.sync 0xffffffff;")
        k("tcgen05.fence::after_thread_sync;")
        k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {ncols};")
        k.mark(end)
        k("ret;")
        return k.render()

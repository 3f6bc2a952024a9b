"""Static shared-memory race check of generated PTX (a sanitizer substitute;
compute-sanitizer's racecheck tool is not available on the pool's GPUs).

The reference ships a symbolic race shadow for its sm_89 output (reference
``tools/checkers/racecheck.py:1-259``): shared-memory addresses are tracked as
``base + a*tid + c``, accesses are grouped into regions between CTA barriers,
and a write/any pair of two different threads in one region that can hit the
same address is a race.  This checker keeps that model and makes it exact
enough for this build's kernels:

* a value is its concrete number in every thread of the launch plus a sum
  of symbolic terms: registers that do not depend on the thread (kernel
  parameters, block indices, loop counters with uniform steps, values loaded
  from uniform addresses) are symbols, so any integer arithmetic on the
  thread index (``tid >> 5``, ``tid & 127``, div/rem, xor swizzles) stays
  exact, and a symbol passes through a shift, div, rem or mask only where it
  provably divides out; two addresses are compared only when their symbolic
  parts are identical, so ``ring + stage*STG + 16*tid`` in two places
  compares exactly;
* an induction register ``v = init; v += step`` (step uniform) is
  ``init + step * iter(v)``, so cooperative strided loops stay exact;
* which threads can execute an access follows from predicates that compare
  thread-affine values with constants (``tid == 0``, ``lane == 0``,
  ``warp < 4``, ...), on the instruction itself and on every branch that
  leads to it (must-facts over the control-flow graph; a loop's exit edge
  adds no fact, every thread that enters a loop leaves it);
* every thread of the launch (``.maxntid``) is enumerated, so a reported race
  names a concrete thread pair and byte address;
* ``bar.sync`` / ``barrier.sync`` / ``barrier.cta`` / ``barrier.cluster.wait``
  start a new region for every thread (a named barrier with a thread count is
  treated as CTA-wide, as the reference does); ``bar.warp.sync`` orders the
  accesses of one warp.

Reported as ``unresolved`` (never as races): accesses whose address mixes
the thread index with a symbol in a way that does not divide out, or whose
guards could not be evaluated; pairs whose symbolic parts differ are not
compared.  Not modelled: asynchronous-proxy traffic (TMA,
``cp.async.bulk``, ``tcgen05``), which the kernels order with mbarriers, and
pairs from different iterations of a barrier-free loop.

``check(ptx, threads=None)`` returns ``(races, stats)``; ``races`` is a list of
``(line_a, line_b, thread_a, thread_b, byte_offset, message)``.
``python -m emmy_b200.racecheck file.ptx ...`` prints them, exits 1 on any.
"""
from __future__ import annotations

import re
import sys
from pathlib import Path

import numpy as np

from .ptxcheck import _blocks, _instructions, _split, _defs_uses

IMM = re.compile(r"^-?(0[xX][0-9a-fA-F]+|\d+)$")
ADDR = re.compile(r"\[\s*([%\w$.]+)\s*(?:\+\s*(-?\w+))?\s*\]")
CTA_BARRIERS = ("bar.sync", "barrier.sync", "bar.red", "barrier.red", "barrier.cta",
                "barrier.cluster.wait", "bar.arrive.sync")
VARYING_SRC = ("%tid", "%laneid", "%warpid", "%clock", "%globaltimer", "%smid")
UNIFORM_SPECIAL = ("%ctaid", "%nctaid", "%ntid", "%cluster", "%nclusterid", "%clusterid",
                   "%is_explicit_cluster")


class Aff:
    """A per-thread integer value: ``arr[t] + sum(coef * symbol)``, the
    symbols uniform (the same in every thread)."""
    __slots__ = ("arr", "u")

    def __init__(self, arr, u=()):
        self.arr = arr
        self.u = tuple(sorted((s, k) for s, k in dict(u).items() if k))

    def __add__(self, o):
        u = dict(self.u)
        for s, k in o.u:
            u[s] = u.get(s, 0) + k
        return Aff(self.arr + o.arr, u)

    def scale(self, k):
        return Aff(self.arr * k, {s: v * k for s, v in self.u})

    def neg(self):
        return self.scale(-1)

    @property
    def uniform(self):
        return bool((self.arr == self.arr[0]).all())

    @property
    def const(self):
        return not self.u and self.uniform

    @property
    def c(self):
        return int(self.arr[0])

    def divisible(self, d):
        return all(k % d == 0 for _, k in self.u)

    def offsets(self, t):
        return self.arr[t]


def _imm(tok):
    return int(tok, 16) if tok.lower().startswith(("0x", "-0x")) else int(tok)


def _operands(rest):
    rest = rest.replace("{", " ").replace("}", " ")
    return [x.strip() for x in rest.split(",") if x.strip()]


class _Kernel:
    def __init__(self, ptx, threads):
        self.ptx = ptx
        self.instrs = _instructions(ptx)
        self.blocks = _blocks(self.instrs)
        m = re.search(r"^\.(?:maxntid|reqntid)\s+(\d+)(?:,\s*(\d+))?(?:,\s*(\d+))?", ptx, re.M)
        dims = [int(x) for x in m.groups() if x] if m else []
        self.tid_yz_zero = len(dims) <= 1 or all(d == 1 for d in dims[1:])
        self.n = threads or (int(np.prod(dims)) if dims else 1024)
        self.t = np.arange(self.n)
        self.defs = {}                       # reg -> [(index, text)]
        self.flat = []                       # (line, text) in order
        for b in self.blocks:
            for ln, text in b["ins"]:
                idx = len(self.flat)
                self.flat.append((ln, text))
                pred, _, op, rest = _split(text)
                d, _ = _defs_uses(op, rest)
                for r in d:
                    self.defs.setdefault(r, []).append((idx, text))
        self.memo = {}
        self.varying = self._varying()

    # ---------------------------------------------------------- uniformity
    def _varying(self):
        """Registers whose value may differ between threads (fixed point)."""
        var = set()
        changed = True
        while changed:
            changed = False
            for r, defs in self.defs.items():
                if r in var:
                    continue
                for _, text in defs:
                    pred, _, op, rest = _split(text)
                    srcs = _operands(rest)[1:]
                    bad = (pred is not None and pred in var)
                    bad |= any(s.startswith(VARYING_SRC) for s in srcs)
                    bad |= op.startswith(("atom", "shfl", "tcgen05.ld", "vote", "match",
                                          "activemask", "redux", "mbarrier"))
                    bad |= any(s in var for s in srcs)
                    if op.startswith("ld") and not bad:
                        m = ADDR.search(rest)
                        bad = bool(m and m.group(1) in var)
                    if bad:
                        var.add(r)
                        changed = True
                        break
        return var

    # -------------------------------------------------------------- values
    def C(self, v=0, u=()):
        return Aff(np.full(self.n, v, dtype=np.int64), u)

    def aff(self, tok):
        tok = tok.strip()
        if IMM.match(tok):
            return self.C(_imm(tok))
        if tok.startswith("%tid.x"):
            return Aff(self.t.copy())
        if tok.startswith(("%tid.y", "%tid.z")):
            return self.C() if self.tid_yz_zero else None
        if tok.startswith("%laneid"):
            return Aff(self.t & 31)
        if tok.startswith(UNIFORM_SPECIAL):
            return self.C(0, {tok: 1})
        if tok.startswith("%"):
            if tok not in self.memo:
                self.memo[tok] = None            # cycle guard
                self.memo[tok] = self._reg_aff(tok)
            return self.memo[tok]
        if re.match(r"^[A-Za-z_$][\w$]*$", tok):
            return self.C(0, {"&" + tok: 1})    # a variable's address
        return None

    def _reg_aff(self, r):
        defs = self.defs.get(r, [])
        if not defs:
            return None
        if len(defs) == 1:
            return self._eval(r, defs[0][1])
        if len(defs) == 2:                       # induction: v = init; v = v + step
            (i0, t0), (i1, t1) = defs
            p1, _, op1, rest1 = _split(t1)
            ops = _operands(rest1)
            if p1 is None and op1.startswith("add") and len(ops) == 3 and ops[1] == r:
                step = self.aff(ops[2])
                if step is not None and step.uniform:
                    self.memo[r] = None
                    init = self._eval(r, t0)
                    if init is not None:
                        key = f"iter({r})"
                        if step.const:
                            return init + self.C(0, {key: step.c})
                        return init + self.C(0, {f"{key}*{ops[2]}": 1})
        if r not in self.varying:
            return self.C(0, {r: 1})
        return None

    def _eval(self, r, text):
        pred, _, op, rest = _split(text)
        ops = _operands(rest)
        base = op.split(".")[0]
        src = ops[1:]
        fallback = self.C(0, {r: 1}) if r not in self.varying else None
        if pred is not None or ".f" in op[len(base):] or ".hi" in op:
            return fallback
        vals = [self.aff(x) for x in src]
        if any(v is None for v in vals):
            return fallback
        try:
            if base in ("mov", "cvta", "cvt") and len(vals) == 1:
                return vals[0]
            if base in ("add", "sub") and len(vals) == 2:
                a, b = vals
                return a + (b if base == "add" else b.neg())
            if base in ("mul", "mad") and len(vals) in (2, 3):
                a, b = vals[:2]
                if b.const:
                    prod = a.scale(b.c)
                elif a.const:
                    prod = b.scale(a.c)
                elif not a.u and not b.u:
                    prod = Aff(a.arr * b.arr)
                else:
                    return fallback
                return prod + vals[2] if base == "mad" else prod
            if base == "shl" and len(vals) == 2 and vals[1].const:
                return vals[0].scale(1 << vals[1].c)
            if base in ("shr", "div", "rem") and len(vals) == 2 and vals[1].const:
                a = vals[0]
                d = (1 << vals[1].c) if base == "shr" else vals[1].c
                if d <= 0 or not a.divisible(d) or (a.arr < 0).any():
                    return fallback
                if base == "rem":
                    return Aff(a.arr % d)
                return Aff(a.arr // d, {s: k // d for s, k in a.u})
            if base == "and" and len(vals) == 2 and vals[1].const:
                a, m = vals[0], vals[1].c
                if not a.u or (m >= 0 and (m + 1) & m == 0 and a.divisible(m + 1)):
                    return Aff(a.arr & m)
            if base in ("or", "xor", "and", "min", "max") and len(vals) == 2 and \
                    not vals[0].u and not vals[1].u:
                a, b = vals[0].arr, vals[1].arr
                f = {"or": np.bitwise_or, "xor": np.bitwise_xor, "and": np.bitwise_and,
                     "min": np.minimum, "max": np.maximum}[base]
                return Aff(f(a, b))
        except (ValueError, IndexError, OverflowError):
            return fallback
        return fallback

    # ---------------------------------------------------------- predicates
    def pmask(self, p):
        """Boolean array over threads where predicate register p holds, or
        'uniform' (same value in every thread), or None (unknown)."""
        if p not in self.varying:
            return "uniform"
        defs = self.defs.get(p, [])
        if len(defs) != 1:
            return None
        pred, _, op, rest = _split(defs[0][1])
        if pred is not None:
            return None
        ops = _operands(rest)
        if op.startswith("setp") and len(ops) >= 3 and "|" not in ops[0]:
            cmp = op.split(".")[1]
            a, b = self.aff(ops[1]), self.aff(ops[2])
            if a is None or b is None:
                return None
            d = a + b.neg()
            if d.u:
                return None
            v = d.arr
            return {"eq": v == 0, "ne": v != 0, "lt": v < 0, "le": v <= 0, "gt": v > 0,
                    "ge": v >= 0, "lo": v < 0, "ls": v <= 0, "hi": v > 0, "hs": v >= 0}.get(cmp)
        if op.startswith(("and.pred", "or.pred", "xor.pred")) and len(ops) == 3:
            a, b = self.pmask(ops[1]), self.pmask(ops[2])
            if a is None or b is None:
                return None
            if isinstance(a, str) or isinstance(b, str):
                return None
            return a & b if op.startswith("and") else a | b if op.startswith("or") else a ^ b
        if op.startswith("not.pred") and len(ops) == 2:
            a = self.pmask(ops[1])
            return ~a if isinstance(a, np.ndarray) else a
        return None

    # -------------------------------------------------------------- guards
    def facts(self):
        """Must-facts per block: {(predicate, polarity)} true on every path."""
        blocks = self.blocks
        start, pos = [], 0
        for b in blocks:
            start.append(pos)
            pos += len(b["ins"])
        label_pos = {b["label"]: start[i] for i, b in enumerate(blocks) if b["label"]}
        loops = []
        for i, b in enumerate(blocks):
            if b["ins"]:
                _, _, op, rest = _split(b["ins"][-1][1])
                tgt = rest.strip()
                if op.startswith("bra") and tgt in label_pos and label_pos[tgt] <= start[i]:
                    loops.append((label_pos[tgt], start[i] + len(b["ins"]) - 1))

        def exits(i, j):
            return any(lo <= start[i] <= hi and not lo <= start[j] <= hi for lo, hi in loops)

        index = {b["label"]: i for i, b in enumerate(blocks) if b["label"]}
        edge = {}
        for i, b in enumerate(blocks):
            last = b["ins"][-1][1] if b["ins"] else ""
            pred, neg, op, rest = _split(last) if last else (None, False, "", "")
            for s in b["succ"]:
                f = frozenset()
                if pred is not None and op.startswith("bra") and not exits(i, s):
                    taken = index.get(rest.strip()) == s
                    f = frozenset({(pred, (not neg) if taken else bool(neg))})
                edge[(i, s)] = f
        preds = [[] for _ in blocks]
        for (i, s) in edge:
            preds[s].append(i)
        top = None
        IN = [top] * len(blocks)
        OUT = [top] * len(blocks)
        IN[0] = frozenset()
        changed = True
        while changed:
            changed = False
            for i in range(len(blocks)):
                if i == 0:
                    new = frozenset()
                else:
                    parts = [OUT[p] | edge[(p, i)] for p in preds[i] if OUT[p] is not None]
                    new = frozenset.intersection(*parts) if parts else None
                if new != IN[i] or new != OUT[i]:
                    IN[i] = OUT[i] = new
                    changed = True
        return IN, start

    def active(self, facts, own):
        """(bool mask over threads, exact?) for an access under these facts."""
        m = np.ones(self.n, dtype=bool)
        exact = True
        for p, pol in list(facts or ()) + ([own] if own else []):
            pm = self.pmask(p)
            if isinstance(pm, str):
                continue
            if pm is None:
                exact = False
                continue
            m &= pm if pol else ~pm
        return m, exact


_WIDTH = {"8": 1, "16": 2, "32": 4, "64": 8, "128": 16}


def _access(op):
    """(kind, bytes) of a generic-proxy shared-memory access, else None."""
    parts = op.split(".")
    base = parts[0]
    if base not in ("ld", "st", "atom", "red") or "shared::cluster" in op:
        return None
    if not any(p == "shared" or p == "shared::cta" for p in parts):
        return None
    vec = 1
    size = 4
    for p in parts[1:]:
        if p.startswith("v") and p[1:].isdigit():
            vec = int(p[1:])
        m = re.match(r"^[bsuf](8|16|32|64|128)$", p) or re.match(r"^bf(16)$", p)
        if m:
            size = _WIDTH[m.group(1)]
    kind = "R" if base == "ld" else "W" if base == "st" else "A"
    return kind, vec * size


def check(ptx: str, threads: int | None = None):
    k = _Kernel(ptx, threads)
    IN, start = k.facts()
    cta_epoch = warp_epoch = 0
    accesses = []
    stats = {"accesses": 0, "unresolved": 0, "threads": k.n}
    idx = 0
    for bi, b in enumerate(k.blocks):
        for ln, text in b["ins"]:
            pred, neg, op, rest = _split(text)
            if op.startswith(CTA_BARRIERS):
                cta_epoch += 1
                warp_epoch += 1
            elif op.startswith("bar.warp.sync"):
                warp_epoch += 1
            acc = _access(op)
            idx += 1
            if acc is None or IN[bi] is None:
                continue
            stats["accesses"] += 1
            m = ADDR.search(rest)
            a = k.aff(m.group(1)) if m else None
            if a is not None and m.group(2):
                try:
                    a = a + k.C(_imm(m.group(2)))
                except ValueError:
                    a = None
            mask, exact = k.active(IN[bi], (pred, not neg) if pred else None)
            if a is None or not exact:
                stats["unresolved"] += 1
                continue
            accesses.append({"line": ln, "text": text, "kind": acc[0], "width": acc[1],
                             "aff": a, "mask": mask, "epoch": cta_epoch, "wepoch": warp_epoch})
    races = []
    groups = {}
    for i, a in enumerate(accesses):
        groups.setdefault((a["epoch"], a["aff"].u), []).append(i)
    seen = set()
    for key, ids in groups.items():
        if not any(accesses[i]["kind"] in "WA" for i in ids):
            continue
        rows = []
        for i in ids:
            a = accesses[i]
            t = k.t[a["mask"]]
            off = a["aff"].offsets(t)
            for j in range(a["width"]):
                rows.append(np.stack([off + j, t, np.full_like(t, i)], axis=1))
        if not rows:
            continue
        allr = np.concatenate(rows)
        order = np.lexsort((allr[:, 1], allr[:, 0]))
        allr = allr[order]
        bytes_ = allr[:, 0]
        cut = np.flatnonzero(np.diff(bytes_)) + 1
        for grp in np.split(allr, cut):
            if len(grp) < 2 or len(np.unique(grp[:, 1])) < 2:
                continue
            kinds = [accesses[x]["kind"] for x in grp[:, 2]]
            if "W" not in kinds and "A" not in kinds:
                continue
            found = None
            for x in range(len(grp)):
                ax = accesses[grp[x, 2]]
                for y in range(x + 1, len(grp)):
                    ay = accesses[grp[y, 2]]
                    tx, ty = int(grp[x, 1]), int(grp[y, 1])
                    if tx == ty or (ax["kind"] == "R" and ay["kind"] == "R"):
                        continue
                    if ax["kind"] == ay["kind"] == "A":
                        continue
                    if tx >> 5 == ty >> 5 and ax["wepoch"] != ay["wepoch"]:
                        continue
                    found = (ax, ay, tx, ty)
                    break
                if found:
                    break
            if found:
                ax, ay, tx, ty = found
                pair = (ax["line"], ay["line"])
                if pair in seen:
                    continue
                seen.add(pair)
                races.append((ax["line"], ay["line"], tx, ty, int(grp[0, 0]),
                              f"{ax['kind']}/{ay['kind']} `{ax['text'][:50]}` vs `{ay['text'][:50]}`"))
    stats["races"] = len(races)
    return races, stats


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    bad = 0
    for f in argv:
        races, stats = check(Path(f).read_text())
        for la, lb, ta, tb, off, msg in races:
            print(f"{f}:{la}:{lb}: race between threads {ta} and {tb} at byte {off}: {msg}")
        bad += len(races)
        print(f"{f}: {stats['accesses']} shared accesses, {stats['unresolved']} unresolved, "
              f"{len(races)} race(s)")
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())

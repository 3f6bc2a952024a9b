"""Static checks of generated PTX: a sanitizer substitute for this build's
kernels (compute-sanitizer is not available on the pool's GPUs).

The reference ships a register definedness/dominance checker over its sm_89
output (reference ``tools/checkers/ptxcheck.py``); this one keeps that check
and adds the rules the sm_100a templates must keep:

* **defined** -- every register an instruction reads is written on every path
  from the entry to it (forward must-be-defined dataflow over the basic
  blocks; a write under a predicate counts only where the register was
  already defined, so ``@p mov r, ..`` alone does not define ``r``);
* **bounded-wait** -- every loop that polls an mbarrier (``try_wait`` /
  ``test_wait``) also reads ``%globaltimer``, i.e. can give up;
* **no-multicast-load** -- no bulk or tensor copy carries a qualifier that
  feeds several CTAs (``broadcast_copy``);
* **tmem** -- a kernel that allocates tensor memory relinquishes the
  allocation permit and deallocates the same number of columns;
* **regsplit** -- ``setmaxnreg`` only together with ``.maxnreg`` and a
  ``// @emmy regsplit`` declaration whose shares fit the launch's registers.

``check(ptx)`` returns a list of findings ``(rule, line number, message)``;
``python -m emmy_b200.ptxcheck file.ptx ...`` prints them and exits 1 if any.
"""
from __future__ import annotations

import re
import sys
from pathlib import Path

REG = re.compile(r"%[A-Za-z_]+\d+\b")
LABEL_DEF = re.compile(r"^(\$?[A-Za-z_][\w$]*):\s*$")
PRED = re.compile(r"^@(!?)(%[A-Za-z_]+\d+)\s+")
# opcodes (first dotted component) that write no register operand
NO_DEF = {"st", "red", "bar", "barrier", "bra", "ret", "exit", "cp", "fence", "prefetch",
          "trap", "membar"}
NO_DEF_FULL = ("mbarrier.init", "mbarrier.arrive", "tcgen05.mma", "tcgen05.commit",
               "tcgen05.st", "tcgen05.alloc", "tcgen05.dealloc", "tcgen05.relinquish",
               "tcgen05.fence", "tcgen05.wait", "setmaxnreg", "griddepcontrol",
               "cp.async", "mbarrier.expect_tx")


def broadcast_copy(op: str) -> bool:
    """A bulk or tensor copy with a qualifier that feeds several CTAs (any
    ``multicast`` form)."""
    return op.startswith("cp.async.bulk") and any(q.startswith("multicast")
                                                  for q in op.split("."))


def _instructions(ptx: str):
    """(line number, text) of each statement inside the entry's body."""
    lines = ptx.splitlines()
    out, inside, depth = [], False, 0
    for n, raw in enumerate(lines, 1):
        s = raw.split("//", 1)[0].strip()
        if not inside:
            if s == "{":
                inside, depth = True, 1
            continue
        if not s:
            continue
        if s.startswith("{"):
            depth += 1
            s = s[1:].strip()
        if s.endswith("}") and not s.endswith("{") and s.count("}") > s.count("{"):
            depth -= 1
            s = s[:-1].strip()
            if depth == 0:
                break
        for part in [p.strip() for p in s.split(";") if p.strip()]:
            if not part.startswith("."):            # .reg / .shared declarations
                out.append((n, part))
    return out


def _split(text):
    """(predicate register or None, negated, opcode, operand string)."""
    m = PRED.match(text)
    pred = neg = None
    if m:
        neg, pred = m.group(1) == "!", m.group(2)
        text = text[m.end():]
    op, _, rest = text.partition(" ")
    return pred, neg, op, rest.strip()


def _defs_uses(op: str, rest: str):
    """Registers an instruction writes and reads."""
    base = op.split(".")[0]
    regs_all = REG.findall(rest)
    if base in NO_DEF or op.startswith(NO_DEF_FULL) or not regs_all:
        return set(), set(regs_all)
    if op.startswith(("mbarrier.try_wait", "mbarrier.test_wait")):
        first = rest.split(",", 1)[0]
        return set(REG.findall(first)), set(REG.findall(rest.split(",", 1)[1]))
    if rest.startswith("{"):
        close = rest.index("}")
        return set(REG.findall(rest[:close])), set(REG.findall(rest[close:]))
    first, _, tail = rest.partition(",")
    # setp / shfl / vote may write "p|q"
    return set(REG.findall(first)), set(REG.findall(tail))


def _blocks(instrs):
    """Basic blocks: list of dicts with label, instructions and successors."""
    blocks, cur = [], {"label": None, "ins": []}
    for n, text in instrs:
        if text.endswith(":") and LABEL_DEF.match(text):
            if cur["ins"] or cur["label"]:
                blocks.append(cur)
            cur = {"label": text[:-1], "ins": []}
            continue
        cur["ins"].append((n, text))
        pred, _, op, rest = _split(text)
        if op.startswith(("bra", "ret", "exit")):
            blocks.append(cur)
            cur = {"label": None, "ins": []}
    if cur["ins"] or cur["label"]:
        blocks.append(cur)
    index = {b["label"]: i for i, b in enumerate(blocks) if b["label"]}
    for i, b in enumerate(blocks):
        succ = []
        last = b["ins"][-1] if b["ins"] else None
        if last:
            pred, _, op, rest = _split(last[1])
            if op.startswith("bra"):
                tgt = rest.strip().rstrip(";")
                if tgt in index:
                    succ.append(index[tgt])
                if pred is not None and i + 1 < len(blocks):
                    succ.append(i + 1)
            elif op.startswith(("ret", "exit")):
                if pred is not None and i + 1 < len(blocks):
                    succ.append(i + 1)
            elif i + 1 < len(blocks):
                succ.append(i + 1)
        elif i + 1 < len(blocks):
            succ.append(i + 1)
        b["succ"] = succ
    return blocks


def _check_defined(blocks, findings):
    n = len(blocks)
    preds = [[] for _ in range(n)]
    for i, b in enumerate(blocks):
        for s in b["succ"]:
            preds[s].append(i)
    universe = set()
    gen = []
    for b in blocks:
        g = set()
        for _, text in b["ins"]:
            pred, _, op, rest = _split(text)
            d, _ = _defs_uses(op, rest)
            universe |= d
            if pred is None:
                g |= d
        gen.append(g)
    IN = [set(universe) for _ in range(n)]
    OUT = [set(universe) for _ in range(n)]
    IN[0] = set()
    changed = True
    while changed:
        changed = False
        for i in range(n):
            if i == 0:
                new_in = set()
            elif preds[i]:
                new_in = set.intersection(*(OUT[p] for p in preds[i]))
            else:
                new_in = set()          # unreachable: nothing is known defined
            new_out = new_in | gen[i]
            if new_in != IN[i] or new_out != OUT[i]:
                IN[i], OUT[i], changed = new_in, new_out, True
    reachable = {0}
    stack = [0]
    while stack:
        i = stack.pop()
        for s in blocks[i]["succ"]:
            if s not in reachable:
                reachable.add(s)
                stack.append(s)
    for i, b in enumerate(blocks):
        if i not in reachable:
            continue
        defined = set(IN[i])
        for ln, text in b["ins"]:
            pred, _, op, rest = _split(text)
            d, u = _defs_uses(op, rest)
            if pred is not None:
                u = u | {pred}
            for r in sorted(u - defined):
                findings.append(("defined", ln, f"{r} read by `{text[:60]}` may be undefined"))
            if pred is None:
                defined |= d


def _check_loops(instrs, findings):
    pos = {}
    for i, (_, text) in enumerate(instrs):
        if text.endswith(":") and LABEL_DEF.match(text):
            pos[text[:-1]] = i
    for i, (ln, text) in enumerate(instrs):
        pred, _, op, rest = _split(text)
        if not op.startswith("bra"):
            continue
        tgt = rest.strip()
        if tgt in pos and pos[tgt] < i:
            body = [t for _, t in instrs[pos[tgt]:i + 1]]
            polls = any("mbarrier.try_wait" in t or "mbarrier.test_wait" in t for t in body)
            if polls and not any("%globaltimer" in t for t in body):
                findings.append(("bounded-wait", ln,
                                 f"loop at {tgt} polls an mbarrier without a time bound"))


def check(ptx: str) -> list:
    findings = []
    instrs = _instructions(ptx)
    _check_defined(_blocks(instrs), findings)
    _check_loops(instrs, findings)
    for n, text in instrs:
        if broadcast_copy(_split(text)[2]):
            findings.append(("no-multicast-load", n, "bulk/tensor copy fed to several CTAs"))
    alloc = re.findall(r"tcgen05\.alloc\.\S+\s+\[[^\]]+\],\s*(\d+)", ptx)
    dealloc = re.findall(r"tcgen05\.dealloc\.\S+\s+%\w+,\s*(\d+)", ptx)
    if alloc:
        if sorted(alloc) != sorted(dealloc):
            findings.append(("tmem", 0, f"tcgen05.alloc {alloc} vs dealloc {dealloc}"))
        if "tcgen05.relinquish_alloc_permit" not in ptx:
            findings.append(("tmem", 0, "allocation permit not relinquished"))
    if "setmaxnreg" in re.sub(r"//.*", "", ptx):
        m = re.search(r"^\.maxnreg (\d+)", ptx, re.M)
        d = re.search(r"^// @emmy regsplit launch=(\d+) threads=(\d+) warpgroups=([\d,]+)$",
                      ptx, re.M)
        if not m or not d:
            findings.append(("regsplit", 0, "setmaxnreg without .maxnreg and a regsplit line"))
        else:
            launch, threads = int(d.group(1)), int(d.group(2))
            shares = [int(x) for x in d.group(3).split(",")]
            if int(m.group(1)) != launch or 128 * sum(shares) > threads * launch:
                findings.append(("regsplit", 0, f"shares {shares} vs {threads} x {launch}"))
            for v in re.findall(r"setmaxnreg\.(?:inc|dec)\.sync\.aligned\.u32 (\d+);", ptx):
                if int(v) not in shares:
                    findings.append(("regsplit", 0, f"setmaxnreg {v} is no declared share"))
    return findings


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    bad = 0
    for f in argv:
        for rule, ln, msg in check(Path(f).read_text()):
            print(f"{f}:{ln}: [{rule}] {msg}")
            bad += 1
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())

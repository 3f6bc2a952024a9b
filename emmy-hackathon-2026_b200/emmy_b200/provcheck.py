"""IR-name -> register provenance check of the statement-by-statement lowering.

The reference checks its own lowering for aliasing (reference
``tools/checkers/provcheck.py:1-164``): it installs a tracking dictionary as
the compiler's name -> register map and flags two IR names bound to one
register unless a known reason (a ``Let`` alias, CSE, a load-cache hit, a
dead value) explains it.  This check instruments ``GenericLowering`` the same
way but asks the question that decides correctness directly: an IR value is
SSA, so a name must keep the value it was bound to.  A violation is

* a name A bound to a register that already holds another name B's value
  (an alias), then
* an instruction that writes that register in place (an ``Accum`` update of
  B, a loop-carried state), then
* a read of A after that write -- later in the program, or in a later
  iteration of a loop that contains both the write and the read and that
  starts after A was bound --

while A is still bound to the register.  A then observes B's new value
instead of its own.  Aliases that are never overwritten, or never read after
the overwrite, are listed as benign.

``check_graph(graph_dict, meta)`` returns ``(violations, aliases, ptx)``;
``python -m emmy_b200.provcheck folder ...`` checks every ``kernel.ir.json``
(with its ``meta.json``) under the folders and exits 1 on any violation.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

from .generic import GenericLowering
from .ptxcheck import _defs_uses, _split


class _Tracked(dict):
    """The lowering's name -> (register, type) map, logging binds and reads
    with the number of PTX lines emitted so far."""

    def __init__(self, owner, init=()):
        super().__init__(init)
        self._owner = owner

    def _pos(self):
        k = getattr(self._owner, "k", None)
        return len(k.lines) if k is not None else 0

    def __setitem__(self, name, val):
        self._owner.prov_log.append(("bind", name, val[0], self._pos()))
        super().__setitem__(name, val)

    def __getitem__(self, name):
        v = super().__getitem__(name)
        self._owner.prov_log.append(("read", name, v[0], self._pos()))
        return v

    def get(self, name, default=None):
        return self[name] if name in self else default


class _ProvLowering(GenericLowering):
    @property
    def vals(self):
        return self._vals

    @vals.setter
    def vals(self, d):
        if not hasattr(self, "prov_log"):
            self.prov_log = []
        self._vals = _Tracked(self, d)


def _writes_and_loops(lines):
    """Per register the PTX line indices that write it; loop line ranges."""
    writes, labels, loops = {}, {}, []
    for i, raw in enumerate(lines):
        s = raw.split("//", 1)[0].strip().rstrip(";").strip()
        if not s:
            continue
        if s.endswith(":"):
            labels[s[:-1]] = i
            continue
        pred, _, op, rest = _split(s)
        d, _ = _defs_uses(op, rest)
        for r in d:
            writes.setdefault(r, []).append(i)
        if op.startswith("bra"):
            tgt = rest.strip()
            if tgt in labels:                    # backward branch: a loop
                loops.append((labels[tgt], i))
    return writes, loops


def analyse(log, lines):
    writes, loops = _writes_and_loops(lines)
    bound = {}                # name -> (reg, bind position)
    holder = {}               # reg -> name whose value it first held
    aliases, violations = [], []
    open_aliases = {}         # name -> (reg, pos, owner)
    for ev, name, reg, pos in log:
        if not isinstance(reg, str) or not reg.startswith("%"):
            if ev == "bind":
                bound.pop(name, None)
                open_aliases.pop(name, None)
            continue
        if ev == "bind":
            prev = bound.get(name)
            owner = holder.setdefault(reg, name)
            bound[name] = (reg, pos)
            open_aliases.pop(name, None)
            if owner != name and not (prev and prev[0] == reg):
                aliases.append((name, owner, reg, pos))
                open_aliases[name] = (reg, pos, owner)
        elif ev == "read" and name in open_aliases:
            reg_a, p0, owner = open_aliases[name]
            if bound.get(name, (None,))[0] != reg_a:
                continue
            for w in writes.get(reg, []):
                if w < p0:
                    continue
                later = w < pos
                looped = any(p0 <= lo <= w <= hi and lo <= pos <= hi for lo, hi in loops)
                if later or looped:
                    violations.append((name, owner, reg, w, pos))
                    open_aliases.pop(name, None)
                    break
    bad = {(v[0], v[2]) for v in violations}
    benign = [a for a in aliases if (a[0], a[2]) not in bad]
    return violations, benign


def check_graph(graph_dict: dict, meta: dict):
    from .context import KernelContext
    from .compiler import find_kernel
    from . import ir as _ir
    g = _ir.load_graph(json.loads(json.dumps(graph_dict)))
    ctx = KernelContext(g, meta, find_kernel(g))
    low = _ProvLowering(ctx)
    low.prov_log = []
    ptx = low.emit()
    violations, benign = analyse(low.prov_log, low.k.lines)
    return violations, benign, ptx


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    bad = 0
    for arg in argv:
        p = Path(arg)
        irs = sorted(p.rglob("kernel.ir.json")) if p.is_dir() else [p]
        for ir in irs:
            meta = ir.parent / "meta.json"
            try:
                v, benign, _ = check_graph(json.loads(ir.read_text()), json.loads(meta.read_text()))
            except NotImplementedError as e:
                print(f"{ir.parent.name}: skipped ({e})")
                continue
            for name, owner, reg, w, r in v:
                print(f"{ir.parent.name}: `{name}` aliases `{owner}` in {reg}, which is "
                      f"overwritten (PTX line {w}) before `{name}` is read (line {r})")
            bad += len(v)
            if not v:
                print(f"{ir.parent.name}: clean ({len(benign)} benign alias(es))")
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env python3
"""Regenerate the golden fixtures under tests/golden/ from the reference tree.

The reference (emmy-hackathon-2026) ships, per open problem, the Kernel IR
(``problems/<id>/*.ir.json``), its launch descriptor (``meta.json``) and the
expected outputs Emmy produced on the seeded inputs (``expected.npz``,
reference ``tools/generate.py:142-151``); and eight bug fixtures with their
raw inputs and frozen outputs (``tests/fixtures/<name>/{in_*.bin,ref.bin}``,
reference ``tests/expectations.json`` "fixtures").  These are test data, not
code: they are copied verbatim (the IR renamed ``kernel.ir.json``) so that the
GPU box, which has no reference tree, can run the parity tests, and a
``MANIFEST.json`` records each file's SHA-256 and origin.

Usage: python tests/golden/make_fixtures.py [--reference <reference checkout>]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
from pathlib import Path

HERE = Path(__file__).resolve().parent


def sha(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EMMY_REFERENCE_ROOT")
                    or str(Path(__file__).resolve().parents[3] / "reference"),
                    help="the reference checkout (default: EMMY_REFERENCE_ROOT, else "
                         "a 'reference' folder beside this repository)")
    args = ap.parse_args()
    ref = Path(args.reference)
    manifest = {}
    for sub in ("problems", "fixtures"):
        d = HERE / sub
        if d.exists():
            shutil.rmtree(d)
        d.mkdir()
    for p in sorted((ref / "problems").iterdir()):
        if not p.is_dir():
            continue
        out = HERE / "problems" / p.name
        out.mkdir()
        irs = sorted(p.glob("*.ir.json"))
        assert len(irs) == 1, p
        pairs = [(irs[0], out / "kernel.ir.json"), (p / "meta.json", out / "meta.json"),
                 (p / "expected.npz", out / "expected.npz")]
        for src, dst in pairs:
            shutil.copyfile(src, dst)
            manifest[str(dst.relative_to(HERE))] = {"from": str(src.relative_to(ref)),
                                                    "sha256": sha(dst)}
    for f in sorted((ref / "tests" / "fixtures").iterdir()):
        out = HERE / "fixtures" / f.name
        out.mkdir()
        for src in sorted(f.iterdir()):
            dst = out / src.name
            shutil.copyfile(src, dst)
            manifest[str(dst.relative_to(HERE))] = {"from": str(src.relative_to(ref)),
                                                    "sha256": sha(dst)}
    (HERE / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"{len(manifest)} files")


if __name__ == "__main__":
    main()

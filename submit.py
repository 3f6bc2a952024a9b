#!/usr/bin/env python3
"""Test a PTX file (or a whole compiler) against one problem, on this GPU.

    python submit.py r01_array_sum out.ptx
    python submit.py r01_array_sum --compiler ./compile.py
    python submit.py path/to/problem_folder --compiler ./compile.py --time

The same command line, messages and exit codes as the reference's ``submit.py``
(reference ``submit.py:53-161``: a usage problem prints its message to stderr and
exits 1, as ``sys.exit(msg)`` does there; argparse's own errors exit 2): with ``--compiler`` every kernel of the problem
is compiled by ``python <compiler> <entry>.ir.json`` in ``meta.json`` order, the
buffers an earlier kernel wrote are handed to later ones (``intermediate``
arguments), and every output named in ``expected.npz`` is compared with
``np.allclose(got, ref, rtol, atol)``.  Instead of a remote runner, the kernels
run on the local B200 through this build's C-ABI runtime.

Exit code 0 = every kernel compiled and the outputs matched within tolerance;
1 = an unknown problem, a missing PTX/--compiler, a multi-kernel problem given
one PTX file, a compiler failure or an output outside tolerance.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "emmy-hackathon-2026_b200"))
PROBLEMS = REPO / "tests" / "golden" / "problems"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("problem", help="problem id, e.g. r01_array_sum, or a problem folder")
    ap.add_argument("ptx", nargs="?", help="a PTX file (single-kernel problems)")
    ap.add_argument("--compiler", help="a compile.py; run once per kernel instead of a PTX file")
    ap.add_argument("--time", action="store_true", help="also time each kernel (CUDA events)")
    args = ap.parse_args(argv)

    pdir = Path(args.problem)
    if not (pdir / "meta.json").exists():
        pdir = PROBLEMS / args.problem
    if not (pdir / "meta.json").exists():
        print(f"unknown problem {args.problem!r}; choose from: "
              + ", ".join(sorted(p.name for p in PROBLEMS.iterdir()
                                 if (p / "meta.json").exists())), file=sys.stderr)
        return 1
    meta = json.loads((pdir / "meta.json").read_text())
    if not args.compiler and not args.ptx:
        print("give a PTX file or --compiler", file=sys.stderr)
        return 1
    if not args.compiler and len(meta["kernels"]) > 1:
        print(f"{args.problem} has {len(meta['kernels'])} kernels - use --compiler",
              file=sys.stderr)
        return 1

    from emmy_b200 import problem
    src = problem.compiler_ptx(args.compiler) if args.compiler else problem.file_ptx(args.ptx)
    report = problem.run_problem(pdir, src, time_launches=args.time)
    return 0 if report["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())

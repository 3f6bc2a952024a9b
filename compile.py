#!/usr/bin/env python3
"""Emmy Kernel IR -> sm_100a PTX.

Contract (unchanged from the reference): ``python compile.py kernel.ir.json > out.ptx``
with ``meta.json`` beside the IR; exit 0 = PTX on stdout, 1 = unsupported
construct, 2 = usage error or missing meta.json.  The compiler lives in the
``emmy_b200`` package; this file keeps the in-process names the reference's
callers import (``Compiler``, ``find_kernel``, ``compile_ir``, ``main``, ``Graph``).
"""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent / "emmy-hackathon-2026_b200"))

from emmy_b200.compiler import Compiler, Graph, compile_ir, find_kernel, main  # noqa: E402,F401

if __name__ == "__main__":
    sys.exit(main())

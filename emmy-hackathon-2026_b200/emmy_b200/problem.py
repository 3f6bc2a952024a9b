"""Problem folders: every kernel of a problem, in ``meta.json`` order, on this GPU.

A problem folder holds one ``<entry>.ir.json`` per kernel, ``meta.json`` and
(for open problems) ``expected.npz`` (reference ``tools/generate.py:74-205``).
The reference's ``submit.py`` (``:60-161``) sends each kernel's PTX to a remote
runner one kernel at a time, feeding buffers written by earlier kernels to later
ones as ``intermediate`` arguments (``:112-122``), and compares every output
named in ``expected.npz`` with ``np.allclose(got, ref, rtol, atol)``
(``:142-158``).  Here the kernels run on the local GPU through the C-ABI
runtime and every buffer stays resident in device memory between kernels, so an
intermediate is simply the same device buffer.

Argument handling follows the reference runner (``tools/harness/gpu_run.py``):
inputs from ``seed`` (``default_rng(seed)``: ``integers(1, 100)`` for integer
dtypes, else ``standard_normal``; this build also reads ``dist``) or ``data``
(broadcast), or ``in_<name>.bin`` in the folder; outputs zero-filled when first
allocated and again before every launch when listed in ``zero_outputs``.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np

from . import harness, native
from .data import bf16_to_f32, materialize


def find_ir(folder: Path, entry: str) -> Path:
    """The kernel's IR file: ``<entry>.ir.json``, or the folder's only IR."""
    p = folder / f"{entry}.ir.json"
    if p.exists():
        return p
    irs = sorted(folder.glob("*.ir.json"))
    if len(irs) == 1:
        return irs[0]
    raise FileNotFoundError(f"no {entry}.ir.json in {folder}")


def compiler_ptx(compiler: str):
    """A PTX source that runs ``python <compiler> <ir.json>`` for each kernel,
    as the reference's ``submit.py --compiler`` does (``:84-92``)."""
    def ptx_for(kernel: dict, ir: Path) -> str:
        r = subprocess.run([sys.executable, compiler, str(ir)], capture_output=True, text=True)
        if r.returncode != 0:
            raise CompileFailed(f"your compiler failed (exit code {r.returncode}):\n"
                                f"{r.stderr or '(nothing on stderr)'}")
        return r.stdout
    return ptx_for


def file_ptx(path: str):
    text = Path(path).read_text()
    return lambda kernel, ir: text


class CompileFailed(RuntimeError):
    pass


def not_ptx(ptx: str) -> str | None:
    """Why this text cannot be PTX, or None."""
    lines = [ln.strip() for ln in ptx.splitlines()
             if ln.strip() and not ln.strip().startswith(("//", "/*", "*"))]
    if not lines:
        return "it is empty"
    if not lines[0].startswith("."):
        return (f"it starts with {lines[0][:60]!r} instead of a directive like .version - "
                "stdout must be PTX only")
    return None


def run_problem(folder, ptx_for=None, out=print, time_launches: bool = False,
                device: str = "cuda", iters: int = 5) -> dict:
    """Run every kernel of the problem in ``folder`` once, in meta order.

    ``ptx_for(kernel_info, ir_path) -> str`` supplies each kernel's PTX; by
    default the kernels are compiled in-process.  Returns ``{"ok": bool,
    "kernels": [...], "outputs": {name: ndarray}}``; ``out`` receives one line
    per checked output (``[entry] PASS name: max abs err ...``).  With
    ``time_launches`` each kernel is also timed, ``iters`` launches back to
    back (CUDA events around each, median), after the checked launch."""
    import torch
    folder = Path(folder)
    meta = json.loads((folder / "meta.json").read_text())
    exp_path = folder / "expected.npz"
    expected = dict(np.load(exp_path)) if exp_path.exists() else {}
    bufs: dict = {}
    args_by_name: dict = {}
    report = {"ok": True, "kernels": [], "outputs": {}}
    stream = torch.cuda.current_stream().cuda_stream
    for k in meta["kernels"]:
        entry = k["entry"]
        ir = find_ir(folder, entry)
        try:
            if ptx_for is None:
                kern = harness.CompiledKernel(json.loads(ir.read_text()), meta)
            else:
                ptx = ptx_for(k, ir)
                if why := not_ptx(ptx):
                    out(f"[{entry}] that is not PTX: {why}")
                    report["ok"] = False
                    return report
                kern = harness.CompiledKernel.from_ptx(ptx, k)
        except (CompileFailed, NotImplementedError, RuntimeError) as e:
            out(f"[{entry}] {e}")
            report["ok"] = False
            return report
        if entry not in kern.image.registers():
            out(f"[{entry}] compiled, but entry points are {sorted(kern.image.registers())} "
                f"- the entry must be named {entry!r}")
            report["ok"] = False
            return report
        ptrs = {}
        for a in k["args"]:
            n = a["name"]
            args_by_name[n] = a
            if a.get("scalar"):
                ptrs[n] = a.get("value", 0)
                continue
            if a.get("output"):
                if n not in bufs:
                    size = max(1, int(np.prod(a["shape"])) if a["shape"] else 1)
                    bufs[n] = torch.zeros(size, dtype=harness.torch_dtype(a["dtype"]),
                                          device=device)
            elif a.get("intermediate"):
                if n not in bufs:
                    out(f"[{entry}] needs {n} from an earlier kernel - kernels run in "
                        f"meta.json order")
                    report["ok"] = False
                    return report
            elif n not in bufs:
                bufs[n] = harness.to_device(materialize(a, folder).reshape(-1), a["dtype"],
                                            device)
            ptrs[n] = bufs[n].data_ptr()
        zero = [(bufs[z].data_ptr(), bufs[z].numel() * bufs[z].element_size())
                for z in k.get("zero_outputs", []) if z in bufs]
        for z, nb in zero:
            native.check(native.lib().emmy_memset_async(z, 0, nb, stream))
        kern.launch(ptrs, stream)
        torch.cuda.synchronize()
        us = None
        if time_launches:
            ms = kern.time(ptrs, warmup=1, iters=iters, stream=stream, zero=zero)
            us = float(np.median(ms)) * 1e3
        report["kernels"].append({"entry": entry, "kind": kern.kind, "us": us})
        for a in k["args"]:
            if not a.get("output"):
                continue
            n = a["name"]
            got = harness.from_device(bufs[n], a["dtype"])
            if a["dtype"] == "bf16":
                got = bf16_to_f32(got)
            report["outputs"][n] = got
            if n not in expected:
                continue
            ref = expected[n]
            g = np.asarray(got).astype(np.float32).reshape(ref.shape)
            err = float(np.max(np.abs(g.astype(np.float64) - ref))) if g.size else 0.0
            tail = f"  ({us:.1f} us)" if us is not None else ""
            if np.allclose(g, ref, rtol=meta["rtol"], atol=meta["atol"]):
                out(f"[{entry}] PASS  {n}: max abs err {err:.3e}{tail}")
            else:
                out(f"[{entry}] FAIL  {n}: max abs err {err:.3e} (tolerance rtol={meta['rtol']} "
                    f"atol={meta['atol']})\n    the parameters must be in meta.json's arg_order: "
                    f"{', '.join(k['arg_order'])}")
                report["ok"] = False
    return report

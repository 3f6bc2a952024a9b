"""Host harness: compile an IR, assemble it, launch it under its meta.json.

This replaces the reference's remote runner and its local ctypes runner
(reference ``submit.py:80-161``, ``tools/harness/gpu_run.py:46-103``) with
the native C-ABI library (:mod:`emmy_b200.native`): PTX is assembled
in-process, loaded into the device's primary context, and launched with
``emmy_launch`` under the meta grid/block/dynamic-smem; outputs named in
``zero_outputs`` are zeroed before every launch (reference
``docs/API.md:52-53``).  Device memory comes from torch (the plumbing); no
torch kernel runs on the measured path.

Kernels that read host-built tensor maps declare them in their PTX with
``// @emmy tmap <param> buf=<arg> dtype=<n> dims=.. strides=.. box=.. swizzle=..``
lines; the harness encodes each one with ``emmy_tensormap_encode`` from the
argument's device address and appends it after the meta ``arg_order``
parameters.
"""
from __future__ import annotations

import ctypes
import json
import os
import re
from pathlib import Path

import numpy as np

from . import native
from .compiler import compile_graph
from .data import NP, materialize, nbytes

_TMAP_RE = re.compile(r"^// @emmy tmap (\S+) (.*)$", re.M)
_CLUSTER_RE = re.compile(r"^// @emmy cluster (\d+) (\d+) (\d+)$", re.M)
_REGSPLIT_RE = re.compile(r"^// @emmy regsplit launch=(\d+) threads=(\d+) warpgroups=([\d,]+)$",
                          re.M)


def check_regsplit(ptx: str, launch_regs: int) -> None:
    """A kernel that moves registers between warpgroups with setmaxnreg may
    only run when the launch holds what the split was computed for: the
    loaded function's register count equal to the declared one, and the
    warpgroup shares adding up to no more than threads x that count
    (otherwise setmaxnreg.inc would wait for registers that never come)."""
    mo = _REGSPLIT_RE.search(ptx)
    if mo is None:
        if "setmaxnreg" in ptx:
            raise RuntimeError("setmaxnreg without a '// @emmy regsplit' declaration")
        return
    want, threads = int(mo.group(1)), int(mo.group(2))
    shares = [int(x) for x in mo.group(3).split(",")]
    if launch_regs != want:
        raise RuntimeError(f"register split expects {want} registers per thread at launch, "
                           f"the loaded function has {launch_regs}")
    if 128 * sum(shares) > threads * want or len(shares) * 128 != threads:
        raise RuntimeError(f"register split {shares} exceeds {threads} x {want}")


def parse_tmaps(ptx: str) -> list:
    out = []
    for m in _TMAP_RE.finditer(ptx):
        kv = dict(p.split("=", 1) for p in m.group(2).split())
        out.append({
            "param": m.group(1), "buf": kv["buf"], "dtype": int(kv["dtype"]),
            "dims": [int(x) for x in kv["dims"].split(",")],
            "strides": [int(x) for x in kv["strides"].split(",")] if kv.get("strides") else [],
            "box": [int(x) for x in kv["box"].split(",")],
            "swizzle": int(kv.get("swizzle", 0)),
            "offset": int(kv.get("offset", 0)),
        })
    return out


def parse_peer(ptx: str) -> list:
    """The trailing cross-GPU parameters a fused full sum declares
    (``// @emmy peer <names>``), in order; none for every other kernel."""
    for line in ptx.splitlines():
        if line.startswith("// @emmy peer "):
            return line.split()[3:]
    return []


def parse_cluster(ptx: str):
    m = _CLUSTER_RE.search(ptx)
    return tuple(int(x) for x in m.groups()) if m else None


class CompiledKernel:
    """One IR compiled to sm_100a PTX, assembled, and (lazily) loaded."""

    def __init__(self, graph_dict: dict, meta: dict, arch: str = "sm_100a"):
        self.graph_dict = graph_dict
        self.meta = meta
        self.compiler = compile_graph(graph_dict, meta)
        self.ptx = self.compiler.render()
        self.kind = self.compiler.kind
        self.ctx = self.compiler.ctx
        self.info = self.ctx.info
        self.image = native.Image(self.ptx, arch)
        self.tmaps = parse_tmaps(self.ptx)
        self.cluster = parse_cluster(self.ptx)
        self.peer_params = parse_peer(self.ptx)
        self._module = None
        self._kernel = None

    @classmethod
    def from_ptx(cls, ptx: str, kernel_info: dict, arch: str = "sm_100a") -> "CompiledKernel":
        """A kernel given as PTX text (a file, another compiler's output),
        launched under one ``meta.json`` kernel entry: parameters in its
        ``arg_order``, scalars from its ``args``, tensor maps if the PTX
        declares any."""
        from types import SimpleNamespace
        self = cls.__new__(cls)
        self.graph_dict = self.meta = self.compiler = None
        self.ptx = ptx
        self.kind = "ptx"
        self.info = kernel_info
        self.ctx = SimpleNamespace(
            entry=kernel_info["entry"], arg_order=list(kernel_info["arg_order"]),
            scalar_tys={a["name"]: a["dtype"] for a in kernel_info.get("args", [])
                        if a.get("scalar")},
            zero_outputs=list(kernel_info.get("zero_outputs", []) or []),
            info=kernel_info)
        self.image = native.Image(ptx, arch)
        self.tmaps = parse_tmaps(ptx)
        self.cluster = parse_cluster(ptx)
        self.peer_params = parse_peer(ptx)
        self._module = None
        self._kernel = None
        return self

    @property
    def entry(self) -> str:
        return self.ctx.entry

    @property
    def grid(self):
        return tuple(self.info["grid"])

    @property
    def block(self):
        return tuple(self.info["block"])

    @property
    def smem(self) -> int:
        return int(self.info.get("smem_bytes", 0) or 0)

    def kernel(self) -> native.KernelHandle:
        if self._kernel is None:
            self._module = native.Module(self.image.data)
            k = self._module.kernel(self.entry)
            check_regsplit(self.ptx, k.attrs()["regs"])
            self._kernel = k
        return self._kernel

    def module(self) -> native.Module:
        self.kernel()
        return self._module

    def params(self, ptrs: dict):
        """cuLaunchKernel parameter array: arg_order values, then tensor maps.
        Returns (void** array, keepalive)."""
        keep = []
        vals = []
        for a in self.ctx.arg_order:
            if a in self.ctx.scalar_tys:
                ty = self.ctx.scalar_tys[a]
                v = ptrs[a]
                c = {"f32": ctypes.c_float, "f64": ctypes.c_double, "i32": ctypes.c_int32,
                     "i64": ctypes.c_int64, "u32": ctypes.c_uint32, "u64": ctypes.c_uint64,
                     "bool": ctypes.c_uint8, "u8": ctypes.c_uint8, "i16": ctypes.c_int16,
                     "u16": ctypes.c_uint16}.get(ty, ctypes.c_uint32)(v)
            else:
                c = ctypes.c_uint64(int(ptrs[a]))
            keep.append(c)
            vals.append(ctypes.cast(ctypes.pointer(c), ctypes.c_void_p))
        for name in self.peer_params:
            # the fused full sum's cross-GPU parameters (peer.FUSED_PARAMS)
            c = (ctypes.c_uint64 if name in ("peer_table", "peer_local") else ctypes.c_uint32)(
                int(ptrs[name]))
            keep.append(c)
            vals.append(ctypes.cast(ctypes.pointer(c), ctypes.c_void_p))
        for t in self.tmaps:
            buf = native.tensormap(t["dtype"], int(ptrs[t["buf"]]) + t["offset"], t["dims"],
                                   t["strides"], t["box"], t["swizzle"])
            keep.append(buf)
            vals.append(ctypes.cast(buf, ctypes.c_void_p))
        arr = (ctypes.c_void_p * max(1, len(vals)))(*vals)
        keep.append(arr)
        return arr, keep

    def _cluster_arg(self):
        return native.u32x3(self.cluster) if self.cluster else None

    def launch(self, ptrs: dict, stream=None) -> None:
        k = self.kernel()
        arr, keep = self.params(ptrs)
        native.check(native.lib().emmy_launch(k.h, native.u32x3(self.grid),
                                              native.u32x3(self.block), self.smem,
                                              self._cluster_arg(), arr, stream))
        del keep

    def time(self, ptrs: dict, *, warmup: int = 3, iters: int = 20, stream=None,
             flush: tuple | None = None, zero: list | None = None) -> np.ndarray:
        """Per-launch device times (ms) from CUDA events, launched by the C-ABI
        library; ``flush`` = (device address, bytes) written between launches,
        ``zero`` = [(address, bytes)] re-zeroed between launches."""
        k = self.kernel()
        arr, keep = self.params(ptrs)
        zero = zero or []
        zd = (ctypes.c_uint64 * max(1, len(zero)))(*[z[0] for z in zero])
        zb = (ctypes.c_size_t * max(1, len(zero)))(*[z[1] for z in zero])
        out = (ctypes.c_float * iters)()
        fd, fb = flush if flush else (0, 0)
        native.check(native.lib().emmy_time_launches(
            k.h, native.u32x3(self.grid), native.u32x3(self.block), self.smem,
            self._cluster_arg(), arr, stream, warmup, iters, fd, fb, zd, zb, len(zero), out))
        del keep
        return np.frombuffer(out, dtype=np.float32).astype(np.float64)


def torch_dtype(dt: str):
    import torch
    return {"f32": torch.float32, "f64": torch.float64, "i32": torch.int32,
            "i64": torch.int64, "f16": torch.float16, "bf16": torch.bfloat16,
            "u8": torch.uint8, "i16": torch.int16, "bool": torch.bool,
            "u16": torch.int16, "u32": torch.int32, "u64": torch.int64}[dt]


def to_device(arr: np.ndarray, dt: str, device):
    import torch
    if dt == "bf16":
        t = torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).view(torch.bfloat16)
    elif dt in ("u16", "u32", "u64"):
        t = torch.from_numpy(np.ascontiguousarray(arr).view({"u16": np.int16, "u32": np.int32,
                                                             "u64": np.int64}[dt]))
    else:
        t = torch.from_numpy(np.ascontiguousarray(arr))
    return t.to(device)


def from_device(t, dt: str) -> np.ndarray:
    import torch
    if dt == "bf16":
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    a = t.cpu().numpy()
    if dt in ("u16", "u32", "u64"):
        a = a.view(NP[dt])
    return a


GUARD_BYTE = 0xA5      # fill of the guard regions around guarded buffers


class Buffers:
    """Device buffers for every meta argument of a kernel (torch-allocated).

    With ``guard`` > 0 (bytes, a multiple of 512 so the data keeps torch's
    alignment) every buffer sits between two guard regions of that size
    filled with ``GUARD_BYTE``, and a copy of every input is kept:
    ``check_guards`` then reports any byte a launch wrote outside an output's
    extent or into an input -- the memory-safety check that stands in for
    compute-sanitizer, which is closed on the GPU pool (the reference runs
    its fixtures under memcheck, ``tools/harness/sanitizer.py:9-30``)."""

    def __init__(self, kern: CompiledKernel, inputs: dict | None = None, folder=None,
                 device="cuda", guard: int = 0):
        import torch
        self.kern = kern
        self.t = {}
        self.args = {a["name"]: a for a in kern.info["args"]}
        inputs = inputs or {}
        for name, a in self.args.items():
            if a.get("scalar"):
                continue
            dt = a["dtype"]
            if a.get("output"):
                n = max(1, int(np.prod(a["shape"])) if a["shape"] else 1)
                self.t[name] = torch.zeros(n, dtype=torch_dtype(dt), device=device)
            else:
                host = inputs[name] if name in inputs else materialize(a, folder)
                self.t[name] = to_device(np.asarray(host).reshape(-1), dt, device)
        self.guard = int(guard)
        self._raw, self._inputs0 = {}, {}
        if self.guard:
            assert self.guard % 512 == 0, "guard regions keep 512-byte alignment"
            for name, t in list(self.t.items()):
                nb = t.numel() * t.element_size()
                raw = torch.full((2 * self.guard + nb,), GUARD_BYTE, dtype=torch.uint8,
                                 device=t.device)
                raw[self.guard:self.guard + nb].copy_(t.view(torch.uint8))
                self._raw[name] = raw
                self.t[name] = raw[self.guard:self.guard + nb].view(t.dtype)
                if not self.args[name].get("output"):
                    self._inputs0[name] = raw[self.guard:self.guard + nb].clone()

    def check_guards(self) -> list:
        """Every violation of a guarded buffer as (argument, where, first
        offending byte offset, bytes changed): ``where`` is "before" or
        "after" for a guard region (offset counted from the region's start)
        and "input" for a changed input byte.  Empty when nothing was
        written out of place."""
        out = []
        g = self.guard
        for name, raw in self._raw.items():
            nb = raw.numel() - 2 * g
            for where, region in (("before", raw[:g]), ("after", raw[g + nb:])):
                bad = (region != GUARD_BYTE).nonzero()
                if bad.numel():
                    out.append((name, where, int(bad[0, 0]), int(bad.shape[0])))
            if name in self._inputs0:
                bad = (raw[g:g + nb] != self._inputs0[name]).nonzero()
                if bad.numel():
                    out.append((name, "input", int(bad[0, 0]), int(bad.shape[0])))
        return out

    @classmethod
    def random(cls, kern: CompiledKernel, seed: int = 0, device="cuda") -> "Buffers":
        """Buffers filled on the device by torch's generator with each input's
        distribution (``dist``; standard normal otherwise) -- for timing runs,
        where values only need the right distribution, not the seed
        convention.  ``data`` arguments keep their exact values."""
        import torch
        self = cls.__new__(cls)
        self.kern = kern
        self.t = {}
        self.args = {a["name"]: a for a in kern.info["args"]}
        g = torch.Generator(device=device).manual_seed(seed)
        for i, (name, a) in enumerate(self.args.items()):
            if a.get("scalar"):
                continue
            n = max(1, int(np.prod(a["shape"])) if a["shape"] else 1)
            dt = torch_dtype(a["dtype"])
            if a.get("output"):
                self.t[name] = torch.zeros(n, dtype=dt, device=device)
            elif "data" in a:
                self.t[name] = to_device(materialize(a).reshape(-1), a["dtype"], device)
            else:
                d = a.get("dist") or {}
                x = torch.empty(n, dtype=torch.float32, device=device)
                if d.get("kind") == "uniform":
                    x.uniform_(float(d.get("lo", 0.0)), float(d.get("hi", 1.0)), generator=g)
                else:
                    x.normal_(0.0, float(d.get("scale", 1.0)), generator=g)
                self.t[name] = x.to(dt)
        return self

    def ptrs(self) -> dict:
        p = {n: t.data_ptr() for n, t in self.t.items()}
        for name, a in self.args.items():
            if a.get("scalar"):
                p[name] = a.get("value", 0)
        return p

    def zero_list(self):
        out = []
        for n in self.kern.ctx.zero_outputs:
            t = self.t[n]
            out.append((t.data_ptr(), t.numel() * t.element_size()))
        return out

    def outputs(self) -> dict:
        res = {}
        for name, a in self.args.items():
            if a.get("output"):
                res[name] = from_device(self.t[name], a["dtype"]).reshape(a["shape"])
        return res


class GuardViolation(RuntimeError):
    """A launch wrote outside its outputs' extents or into an input."""


def guard_bytes() -> int:
    """Guard-region size for ``run`` from ``EMMY_GUARD_BYTES`` (0: none).
    The test suite sets it, so every launch it makes through ``run`` is
    checked for out-of-place writes (the role of the reference's
    ``EMMY_SANITIZER``, ``tools/harness/sanitizer.py:19``, which runs the
    launch under compute-sanitizer's memcheck)."""
    v = os.environ.get("EMMY_GUARD_BYTES", "").strip()
    return int(v) if v else 0


def run(graph_dict: dict, meta: dict, inputs: dict | None = None, folder=None,
        device="cuda", kern: CompiledKernel | None = None):
    """Compile + launch once; returns ({output: ndarray}, CompiledKernel).
    Under ``EMMY_GUARD_BYTES`` the buffers are guarded and a launch that
    wrote out of place raises ``GuardViolation``."""
    kern = kern or CompiledKernel(graph_dict, meta)
    outs, kern, bad = run_guarded(graph_dict, meta, inputs, folder, guard_bytes(), kern, device)
    if bad:
        raise GuardViolation(f"{kern.ctx.entry}: bytes written out of place "
                             f"(argument, where, first offset, count): {bad}")
    return outs, kern


def run_guarded(graph_dict: dict, meta: dict, inputs: dict | None = None, folder=None,
                guard: int = 1 << 16, kern: CompiledKernel | None = None, device="cuda"):
    """Compile + launch once with every buffer between guard regions of
    ``guard`` bytes (0: plain buffers): returns ({output: ndarray},
    CompiledKernel, violations) -- the violations as
    ``Buffers.check_guards`` lists them, read after the launch."""
    import torch
    kern = kern or CompiledKernel(graph_dict, meta)
    bufs = Buffers(kern, inputs, folder, device, guard=guard)
    stream = torch.cuda.current_stream().cuda_stream
    for z, nb in bufs.zero_list():
        native.check(native.lib().emmy_memset_async(z, 0, nb, stream))
    kern.launch(bufs.ptrs(), stream)
    torch.cuda.synchronize()
    return bufs.outputs(), kern, bufs.check_guards()


def load_problem(folder) -> tuple[dict, dict]:
    folder = Path(folder)
    irs = sorted(folder.glob("*.ir.json"))
    return json.loads(irs[0].read_text()), json.loads((folder / "meta.json").read_text())


def run_host(kern: CompiledKernel, host: dict, dev: dict, stream=None,
             resident=()) -> None:
    """The reference-facing round trip through ``emmy_run_host``: host inputs
    copied in, outputs zeroed, one launch, host outputs copied back.  ``host``
    and ``dev`` map arg names to numpy arrays / torch device tensors; inputs
    named in ``resident`` already hold their data on the device (an earlier
    call of the same step copied them) and are passed with 0 bytes to copy."""
    k = kern.kernel()
    names = kern.ctx.arg_order
    args = {a["name"]: a for a in kern.info["args"]}
    n = len(names)
    hp = (ctypes.c_void_p * n)(*[host[x].ctypes.data for x in names])
    dp = (ctypes.c_uint64 * n)(*[dev[x].data_ptr() for x in names])
    nb = (ctypes.c_size_t * n)(*[0 if (x in resident and not args[x].get("output"))
                                 else nbytes(args[x]) for x in names])
    io = (ctypes.c_int * n)(*[1 if args[x].get("output") else 0 for x in names])
    extra = []
    keep = []
    if kern.tmaps:
        arr, keep = kern.params({x: dev[x].data_ptr() for x in names})
        extra = [arr[i] for i in range(n, n + len(kern.tmaps))]
    ex = (ctypes.c_void_p * max(1, len(extra)))(*extra) if extra else None
    native.check(native.lib().emmy_run_host(
        k.h, native.u32x3(kern.grid), native.u32x3(kern.block), kern.smem,
        kern._cluster_arg(), n, hp, dp, nb, io, len(extra), ex, stream))
    del keep

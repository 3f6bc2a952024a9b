"""PTX text builder for the sm_100a kernel templates.

A :class:`Kernel` collects the body lines of one ``.entry``, hands out typed
virtual registers (ptxas does the real allocation) and renders the module:
``.version 8.8`` / ``.target sm_100a`` header, module-scope declarations, the
entry signature in meta ``arg_order`` (buffers as ``.param .u64``, scalar
arguments by value; reference ``compile.py:2560-2569``) and the register
declarations.  PTX must be ASCII only (reference ``TASK.md:200``);
:meth:`Kernel.render` checks that.
"""
from __future__ import annotations

import struct

PTX_VERSION = "8.8"
TARGET = "sm_100a"

# register class -> PTX declaration type
_REG_DECL = {"p": "pred", "f": "f32", "fd": "f64", "r": "b32", "rd": "b64", "h": "b16", "q": "b128"}

# graph dtype -> (register class, PTX scalar type for ld/st/cvt)
DTYPES = {
    "f32": ("f", "f32"), "f64": ("fd", "f64"), "i32": ("r", "s32"), "i64": ("rd", "s64"),
    "u32": ("r", "u32"), "u64": ("rd", "u64"), "bool": ("r", "u32"),
    "u8": ("r", "u8"), "u16": ("r", "u16"), "i16": ("r", "s16"),
    "f16": ("h", "f16"), "bf16": ("h", "bf16"),
}

# scalar (by-value) kernel arguments are declared with these PTX param types
# (reference compile.py:2564-2566: f16 -> b16, bool -> u8)
PARAM_TYPES = {"f32": "f32", "f64": "f64", "i32": "s32", "i64": "s64", "u32": "u32",
               "u64": "u64", "bool": "u8", "u8": "u8", "u16": "u16", "i16": "s16",
               "f16": "b16", "bf16": "b16"}


def f32_hex(v: float) -> str:
    """Exact PTX spelling of an f32 constant (``0fXXXXXXXX``)."""
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", float(v)))[0]


def f64_hex(v: float) -> str:
    return "0d%016X" % struct.unpack("<Q", struct.pack("<d", float(v)))[0]


class Kernel:
    def __init__(self, entry: str, params, *, version: str = PTX_VERSION,
                 target: str = TARGET):
        """``params``: list of ``(name, ptx_param_type)``; pointer buffers use
        ``"u64"``.  Extra trailing parameters (e.g. 128-byte tensor maps) are
        given as ``(name, ".align 64 .b8", "[128]")`` triples."""
        self.entry = entry
        self.params = list(params)
        self.version = version
        self.target = target
        self.lines: list[str] = []
        self.counts: dict[str, int] = {}
        self.decls: list[str] = []
        self.directives: list[str] = []
        self.label_n = 0
        self.maxntid = None
        self.maxnreg = None
        self.minnctapersm = None
        self.reqnctapercluster = None

    # registers / labels ------------------------------------------------
    def reg(self, cls: str) -> str:
        n = self.counts.get(cls, 0) + 1
        self.counts[cls] = n
        return f"%{cls}{n}"

    def regs(self, cls: str, n: int) -> list[str]:
        return [self.reg(cls) for _ in range(n)]

    def label(self, base: str = "L") -> str:
        self.label_n += 1
        return f"$L_{base}_{self.label_n}"

    # body --------------------------------------------------------------
    def emit(self, *lines: str) -> None:
        for ln in lines:
            self.lines.append("\t" + ln)

    def __call__(self, *lines: str) -> None:
        self.emit(*lines)

    def mark(self, label: str) -> None:
        self.lines.append(f"{label}:")

    def comment(self, text: str) -> None:
        self.lines.append("\t// " + text)

    def decl(self, text: str) -> None:
        """Module-scope declaration (``.shared``/``.global`` variables)."""
        self.decls.append(text)

    def directive(self, text: str) -> None:
        """An ``// @emmy ...`` line the host harness reads (e.g. tensor maps)."""
        self.directives.append(f"// @emmy {text}")

    # constants -----------------------------------------------------------
    def param_ptr(self, name: str) -> str:
        """Load a pointer parameter and convert it to a global address."""
        p = self.reg("rd")
        self.emit(f"ld.param.u64 {p}, [param_{name}];")
        g = self.reg("rd")
        self.emit(f"cvta.to.global.u64 {g}, {p};")
        return g

    def special(self, sreg: str) -> str:
        r = self.reg("r")
        self.emit(f"mov.u32 {r}, {sreg};")
        return r

    # render --------------------------------------------------------------
    def render(self) -> str:
        out = [f".version {self.version}", f".target {self.target}", ".address_size 64", ""]
        out.extend(self.directives)
        if self.directives:
            out.append("")
        out.extend(self.decls)
        if self.decls:
            out.append("")
        out.append(f".visible .entry {self.entry}(")
        ps = []
        for p in self.params:
            if len(p) == 3:
                ps.append(f"\t.param {p[1]} param_{p[0]}{p[2]}")
            else:
                ps.append(f"\t.param .{p[1]} param_{p[0]}")
        out.append(",\n".join(ps))
        out.append(")")
        perf = []
        if self.maxntid:
            perf.append(".maxntid " + ", ".join(str(x) for x in self.maxntid))
        if self.maxnreg:
            perf.append(f".maxnreg {self.maxnreg}")
        if self.minnctapersm:
            perf.append(f".minnctapersm {self.minnctapersm}")
        if self.reqnctapercluster:
            perf.append(".reqnctapercluster " + ", ".join(str(x) for x in self.reqnctapercluster))
        out.extend(perf)
        out.append("{")
        for cls in sorted(self.counts):
            out.append(f"\t.reg .{_REG_DECL[cls]} %{cls}<{self.counts[cls] + 1}>;")
        out.extend(self.lines)
        out.append("}")
        text = "\n".join(out) + "\n"
        if not text.isascii():
            raise ValueError("PTX must be ASCII only")
        return text

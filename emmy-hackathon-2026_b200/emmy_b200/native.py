"""ctypes binding of the C-ABI runtime ``libemmy_b200.so`` (include/emmy_b200.h).

The library is built in-tree by :func:`build` (``g++`` over
``csrc/emmy_runtime.cpp`` with the toolkit's static nvPTXCompiler, so ptxas
runs in-process).  Every wrapper raises :class:`EmmyError` with the
library's ``emmy_last_error()`` text when a call fails; there is no fallback
path -- if the library is missing, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
REPO = ROOT.parent
LIB_PATH = PKG / "libemmy_b200.so"
SRC = ROOT / "csrc" / "emmy_runtime.cpp"
NOALLOC_SRC = ROOT / "csrc" / "emmy_noalloc.cu"
HEADER = REPO / "include" / "emmy_b200.h"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

# exported symbols, in the order include/emmy_b200.h declares them
EXPORTS = [
    "emmy_abi_version", "emmy_last_error", "emmy_ptx_assemble", "emmy_image_data",
    "emmy_image_log", "emmy_image_free", "emmy_device_count", "emmy_device_init",
    "emmy_module_load", "emmy_module_unload", "emmy_kernel_get", "emmy_kernel_attrs",
    "emmy_module_global", "emmy_tensormap_encode", "emmy_launch", "emmy_memset_async",
    "emmy_memcpy_htod_async", "emmy_memcpy_dtoh_async", "emmy_stream_sync", "emmy_mem_alloc",
    "emmy_mem_free", "emmy_ipc_handle", "emmy_ipc_open", "emmy_ipc_close",
    "emmy_time_launches", "emmy_run_host", "emmy_rmsnorm_noalloc",
]


class EmmyError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the runtime library in-tree (host C++ only; the GPU code is the
    PTX each IR compiles to)."""
    deps = [SRC, NOALLOC_SRC, HEADER]
    if LIB_PATH.exists() and not force and all(
            LIB_PATH.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB_PATH
    inc = CUDA_HOME / "include"
    ptxc = CUDA_HOME / "lib64" / "libnvptxcompiler_static.a"
    tmp = LIB_PATH.with_suffix(".so.tmp")
    # the no-allocation entry point holds its scratch in a __device__ array:
    # its one .cu file is compiled by nvcc for sm_100a, with the CUDA runtime
    # linked statically
    obj = LIB_PATH.with_suffix(".noalloc.o")
    r = subprocess.run([str(CUDA_HOME / "bin" / "nvcc"), "-c", "-O2", "-std=c++17",
                        "-gencode", "arch=compute_100a,code=sm_100a",
                        "-Xcompiler", "-fPIC,-fvisibility=hidden", str(NOALLOC_SRC),
                        "-o", str(obj)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compiling {NOALLOC_SRC.name} failed:\n{r.stderr[-4000:]}")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wextra",
           "-fvisibility=hidden", "-Wl,--exclude-libs,ALL", "-s",
           f"-I{inc}", str(SRC), str(obj), "-o", str(tmp), str(ptxc),
           f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    obj.unlink(missing_ok=True)
    if r.returncode != 0:
        raise RuntimeError(f"building {LIB_PATH.name} failed:\n{r.stderr[-4000:]}")
    if verbose and r.stderr:
        print(r.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is not built; run __graft_entry__.build() (no fallback exists)")
        L = ctypes.CDLL(str(LIB_PATH))
        c_u32p = ctypes.POINTER(ctypes.c_uint32)
        L.emmy_last_error.restype = ctypes.c_char_p
        L.emmy_image_log.restype = ctypes.c_char_p
        L.emmy_ptx_assemble.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                        ctypes.POINTER(ctypes.c_char_p), ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_void_p)]
        L.emmy_image_data.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                      ctypes.POINTER(ctypes.c_size_t)]
        L.emmy_image_log.argtypes = [ctypes.c_void_p]
        L.emmy_image_free.argtypes = [ctypes.c_void_p]
        L.emmy_image_free.restype = None
        L.emmy_module_load.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.POINTER(ctypes.c_void_p)]
        L.emmy_module_unload.argtypes = [ctypes.c_void_p]
        L.emmy_kernel_get.argtypes = [ctypes.c_void_p, ctypes.c_char_p,
                                      ctypes.POINTER(ctypes.c_void_p)]
        L.emmy_kernel_attrs.argtypes = [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_int)] * 3
        L.emmy_module_global.argtypes = [ctypes.c_void_p, ctypes.c_char_p,
                                         ctypes.POINTER(ctypes.c_uint64),
                                         ctypes.POINTER(ctypes.c_size_t)]
        L.emmy_tensormap_encode.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64),
                                            ctypes.POINTER(ctypes.c_uint64), c_u32p,
                                            ctypes.c_int]
        L.emmy_launch.argtypes = [ctypes.c_void_p, c_u32p, c_u32p, ctypes.c_uint32, c_u32p,
                                  ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        L.emmy_memset_async.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_size_t,
                                        ctypes.c_void_p]
        L.emmy_memcpy_htod_async.argtypes = [ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.c_void_p]
        L.emmy_memcpy_dtoh_async.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t,
                                             ctypes.c_void_p]
        L.emmy_stream_sync.argtypes = [ctypes.c_void_p]
        L.emmy_mem_alloc.argtypes = [ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t]
        L.emmy_mem_free.argtypes = [ctypes.c_uint64]
        L.emmy_ipc_handle.argtypes = [ctypes.c_uint64, ctypes.c_char_p]
        L.emmy_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]
        L.emmy_ipc_close.argtypes = [ctypes.c_uint64]
        L.emmy_device_count.argtypes = [ctypes.POINTER(ctypes.c_int)]
        L.emmy_device_init.argtypes = [ctypes.c_int]
        L.emmy_time_launches.argtypes = [ctypes.c_void_p, c_u32p, c_u32p, ctypes.c_uint32, c_u32p,
                                         ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                         ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64),
                                         ctypes.POINTER(ctypes.c_size_t), ctypes.c_int,
                                         ctypes.POINTER(ctypes.c_float)]
        L.emmy_run_host.argtypes = [ctypes.c_void_p, c_u32p, c_u32p, ctypes.c_uint32, c_u32p,
                                    ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                    ctypes.POINTER(ctypes.c_uint64),
                                    ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_int),
                                    ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                    ctypes.c_void_p]
        L.emmy_rmsnorm_noalloc.argtypes = [ctypes.c_void_p, c_u32p, c_u32p, ctypes.c_void_p,
                                           c_u32p, c_u32p] + [ctypes.c_uint64] * 5 + [
                                           ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        _LIB = L
    return _LIB


def check(rc: int) -> None:
    if rc != 0:
        raise EmmyError(rc, lib().emmy_last_error().decode(errors="replace"))


def u32x3(v) -> ctypes.Array:
    v = list(v) + [1] * (3 - len(v))
    return (ctypes.c_uint32 * 3)(*v[:3])


class Image:
    """An assembled cubin (ptxas in-process)."""

    def __init__(self, ptx: str, arch: str = "sm_100a", opts=()):
        L = lib()
        h = ctypes.c_void_p()
        raw = ptx.encode()
        arr = (ctypes.c_char_p * max(1, len(opts)))(*[o.encode() for o in opts])
        check(L.emmy_ptx_assemble(raw, len(raw), arch.encode(), arr, len(opts), ctypes.byref(h)))
        self.h = h
        data = ctypes.c_void_p()
        n = ctypes.c_size_t()
        check(L.emmy_image_data(h, ctypes.byref(data), ctypes.byref(n)))
        self.data = ctypes.string_at(data, n.value)
        self.log = L.emmy_image_log(h).decode(errors="replace")

    def __del__(self):
        try:
            lib().emmy_image_free(self.h)
        except Exception:
            pass

    def registers(self) -> dict:
        """Registers per entry from ptxas's info log."""
        import re
        out, cur = {}, None
        for ln in self.log.splitlines():
            m = re.search(r"Compiling entry function '([^']+)'", ln)
            if m:
                cur = m.group(1)
            m = re.search(r"Used (\d+) registers", ln)
            if m and cur:
                out[cur] = int(m.group(1))
        return out


class Module:
    def __init__(self, image: bytes):
        L = lib()
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(image, len(image))
        check(L.emmy_module_load(buf, len(image), ctypes.byref(h)))
        self.h = h

    def kernel(self, entry: str) -> "KernelHandle":
        h = ctypes.c_void_p()
        check(lib().emmy_kernel_get(self.h, entry.encode(), ctypes.byref(h)))
        return KernelHandle(h)

    def global_addr(self, name: str):
        p = ctypes.c_uint64()
        n = ctypes.c_size_t()
        check(lib().emmy_module_global(self.h, name.encode(), ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def unload(self):
        if self.h:
            check(lib().emmy_module_unload(self.h))
            self.h = None


class KernelHandle:
    def __init__(self, h):
        self.h = h

    def attrs(self) -> dict:
        r, s, t = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(lib().emmy_kernel_attrs(self.h, ctypes.byref(r), ctypes.byref(s), ctypes.byref(t)))
        return {"regs": r.value, "static_smem": s.value, "max_threads": t.value}


def device_count() -> int:
    n = ctypes.c_int()
    rc = lib().emmy_device_count(ctypes.byref(n))
    return n.value if rc == 0 else 0


def tensormap(dtype: int, gaddr: int, dims, strides, box, swizzle: int) -> ctypes.Array:
    """One 128-byte CUtensorMap (innermost dimension first)."""
    buf = (ctypes.c_uint8 * 128)()
    rank = len(dims)
    d = (ctypes.c_uint64 * rank)(*dims)
    s = (ctypes.c_uint64 * max(1, rank - 1))(*(list(strides) or [0]))
    b = (ctypes.c_uint32 * rank)(*box)
    check(lib().emmy_tensormap_encode(buf, dtype, rank, gaddr, d, s, b, swizzle))
    return buf

"""Launch arguments: dtypes and how input buffers are filled.

The reference runner fills inputs from the meta argument forms
(reference ``docs/API.md:42-53``, ``tools/harness/gpu_run.py:27-43``):

* ``"seed": s``   -> ``np.random.default_rng(s).standard_normal(shape)`` cast to
  the dtype (integer dtypes: ``rng.integers(1, 100)``);
* ``"data": [..]`` -> the listed values (constants arrive this way), broadcast
  to the shape;
* ``"output": true`` -> allocated zero-filled;
* an ``in_<name>.bin`` file next to the IR (bug fixtures) -> its raw bytes.

This module adds one optional form for the benchmark configurations,
``"dist": {"kind": "uniform", "lo": a, "hi": b}`` or ``{"kind": "normal",
"scale": c}``, drawn from ``default_rng(seed)``.  ``bf16`` buffers are the
round-to-nearest-even bfloat16 of the f32 draw, held as ``uint16`` bits.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

NP = {"f32": np.float32, "f64": np.float64, "i32": np.int32, "i64": np.int64,
      "u32": np.uint32, "u64": np.uint64, "i16": np.int16, "u16": np.uint16,
      "u8": np.uint8, "bool": np.bool_, "f16": np.float16, "bf16": np.uint16}
NBYTES = {k: np.dtype(v).itemsize for k, v in NP.items()}


def nelem(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def nbytes(arg) -> int:
    return max(nelem(arg["shape"]) * NBYTES.get(arg["dtype"], 4), 4)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def materialize(arg: dict, folder: Path | None = None) -> np.ndarray:
    """Host contents of one input buffer (shape ``arg['shape']``)."""
    shape = tuple(int(s) for s in arg["shape"])
    dt = arg["dtype"]
    n = nelem(shape)
    if folder is not None:
        f = Path(folder) / f"in_{arg['name']}.bin"
        if f.exists():
            raw = np.fromfile(f, dtype=np.uint8)[: n * NBYTES.get(dt, 4)]
            return raw.view(NP.get(dt, np.uint8)).reshape(shape)
    if "data" in arg:
        vals = np.asarray(arg["data"], dtype=np.float64)
        flat = np.resize(vals, n) if vals.size else np.zeros(n)
        if dt == "bf16":
            return bf16_bits(flat.astype(np.float32)).reshape(shape)
        return flat.astype(NP.get(dt, np.float32)).reshape(shape)
    if arg.get("output"):
        return np.zeros(shape, dtype=NP.get(dt, np.float32))
    rng = np.random.default_rng(arg.get("seed", 0))
    dist = arg.get("dist")
    npdt = np.dtype(NP.get(dt, np.float32))
    if dt != "bf16" and npdt.kind in "iu":
        return rng.integers(1, 100, size=shape).astype(npdt)
    if dist and dist.get("kind") == "uniform":
        x = rng.uniform(float(dist.get("lo", 0.0)), float(dist.get("hi", 1.0)), size=shape)
    else:
        # float64 draw, then cast: the reference's exact sequence
        x = rng.standard_normal(shape)
        if dist and "scale" in dist:
            x = x * float(dist["scale"])
    if dt == "bf16":
        return bf16_bits(np.asarray(x, dtype=np.float32))
    return np.asarray(x).astype(npdt)

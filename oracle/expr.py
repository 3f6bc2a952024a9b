"""CPU oracle for the five kernel categories -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import this module; the product (``compile.py`` and the ``emmy_b200``
package) never does.

The reference checks every kernel against a numpy/torch evaluation of the
kernel's PyTorch expression on the seeded inputs: Emmy's generator evaluates
it and stores ``expected.npz`` (reference ``tools/generate.py:142-151``), the
open-set expression table pairs each expression with a float64 numpy
reference cast to float32 (``tools/expressions_open.py:52-104``), and the
corpus oracles are numpy lambdas (``tools/harness/refs.py:22-124``).  This
module restates those evaluations:

* float64 arithmetic on the inputs, cast to float32 at the end, for
  reductions, fused row ops, matmul and attention;
* float32 arithmetic in the IR's operation order for pointwise kernels, which
  is what "bit-exact vs numpy" means for ``a + b`` and ``x * c + d``.

Pinned by ``tests/test_oracle.py``: every open problem's ``expected.npz``
(all five categories) is reproduced within the problem's own rtol/atol.
"""
from __future__ import annotations

import numpy as np

f32, f64 = np.float32, np.float64


def _d(x):
    return np.asarray(x, dtype=f64)


# --------------------------------------------------------------------------
# expression families (float64 unless noted)
# --------------------------------------------------------------------------

def add_f32(a, b):
    """``a + b`` in float32 (one ``add.rn.f32`` per element)."""
    return np.add(np.asarray(a, f32), np.asarray(b, f32), dtype=f32)


def scale_shift_f32(x, m, c):
    """``x * m + c`` in float32, two roundings (reference p02, ops multiply then add)."""
    return np.add(np.multiply(np.asarray(x, f32), f32(m), dtype=f32), f32(c), dtype=f32)


def relu_mul_f32(x, y):
    return np.multiply(np.asarray(y, f32), np.maximum(np.asarray(x, f32), f32(0)), dtype=f32)


def full_sum(x):
    return np.asarray(_d(x).sum(), dtype=f32)


def full_mean(x):
    return np.asarray(_d(x).mean(), dtype=f32)


def row_sum(x):
    return _d(x).sum(-1).astype(f32)


def row_mean(x):
    return _d(x).mean(-1).astype(f32)


def rmsnorm(x, w, eps):
    """``x * rsqrt(mean(x^2) + eps) * w`` (reference f01 with its eps)."""
    x = _d(x)
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return (x * r * _d(w)).astype(f32)


def softmax_rows(x, scale=1.0):
    """Row softmax of ``scale * x`` (reference f02; the benchmark scales by 4)."""
    z = _d(x) * scale
    z = z - z.max(-1, keepdims=True)
    e = np.exp(z)
    return (e / e.sum(-1, keepdims=True)).astype(f32)


def l2norm(x, eps=None):
    """``x / ||x||_2`` per row; with ``eps``, ``x / max(||x||_2, eps)`` (F.normalize)."""
    x = _d(x)
    n = np.sqrt((x * x).sum(-1, keepdims=True))
    if eps is not None:
        n = np.maximum(n, eps)
    return (x / n).astype(f32)


def matmul(a, b):
    return (_d(a) @ _d(b)).astype(f32)


def attention(q, k, v, scale, k_transposed=False):
    """``softmax(q k^T * scale) v`` per leading (batch, head) index, float64.
    ``k_transposed``: ``k`` is given as ``k^T`` (the reference's open problems
    pre-transpose it, ``tools/expressions_open.py:91-92``)."""
    q, k, v = _d(q), _d(k), _d(v)
    kt = k if k_transposed else np.swapaxes(k, -1, -2)
    s = (q @ kt) * scale
    s = s - s.max(-1, keepdims=True)
    e = np.exp(s)
    p = e / e.sum(-1, keepdims=True)
    return (p @ v).astype(f32)


# --------------------------------------------------------------------------
# IR nodes the vocabulary defines and no reference IR uses, restated from
# their descriptions in the reference's TASK.md (Pre / Carry, Select,
# ZeroPrologue); the IRs are synth.carried_prefix / select_branches /
# zero_prologue
# --------------------------------------------------------------------------

def carried_prefix(x, every):
    """A carried cell stepped along each row: step j reads the previous state
    (0 before the first step), and steps with j % every == 0 set it to that
    state + x[j]; the output of step j is the state the step read."""
    x = _d(x)
    y = np.zeros_like(x)
    state = np.zeros(x.shape[0])
    for j in range(x.shape[1]):
        y[:, j] = state
        if j % every == 0:
            state = state + x[:, j]
    return y.astype(f32)


def select_split(x, split):
    """The value of the branch whose coordinate predicate holds: x[i] for
    i < split, x[i] * x[i] (float32) otherwise."""
    x = np.asarray(x, f32)
    i = np.arange(x.shape[0])
    return np.where(i < split, x, np.multiply(x, x, dtype=f32)).astype(f32)


def zero_prologue(x, words):
    """The first ``words`` words zeroed, then x added into the first n."""
    x = np.asarray(x, f32)
    out = np.zeros(max(words, x.shape[0]), f32)
    out[:x.shape[0]] += x
    return out


def mma_matmul(a, b, b_kn=True, bias=None, tf32=False, out_bf16=False):
    """C = A . B (B given [K, N], or [N, K] when not ``b_kn``) in float64,
    then relu(C + bias[col]) when a bias is given, as float32 (bf16-rounded
    when the output buffer is bf16).  tf32 operands: each input rounded to
    tf32 (10 explicit mantissa bits, round to nearest, ties away; or
    truncated when ``tf32 == "trunc"``) first."""
    a, b = _d(a), _d(b)
    if tf32:
        a, b = _tf32(a, tf32 == "trunc"), _tf32(b, tf32 == "trunc")
    c = a @ (b if b_kn else b.T)
    if bias is not None:
        c = np.maximum(c + _d(bias)[None, :], 0.0)
    c = c.astype(f32)
    if out_bf16:
        c = bf16_to_f32(bf16_bits_rn(c))
    return c


def mma_attention(q, k, v, scale, causal=False, bias=None):
    """softmax(Q K^T * scale (+ bias), keys after the query masked when
    causal) V in float64, as float32."""
    q, k, v = _d(q), _d(k), _d(v)
    s = (q @ k.T) * scale
    if bias is not None:
        s = s + _d(bias) * 1.0
    if causal:
        i = np.arange(s.shape[0])[:, None]
        j = np.arange(s.shape[1])[None, :]
        s = np.where(j <= i, s, -np.inf)
    s = s - s.max(-1, keepdims=True)
    e = np.exp(s)
    return ((e / e.sum(-1, keepdims=True)) @ v).astype(f32)


def _tf32(x, trunc=False):
    """Round float32 values to tf32: keep the top 10 mantissa bits, round to
    nearest with ties away from zero (PTX cvt.rna.tf32.f32); ``trunc``: drop
    the low 13 bits instead (a tensor core reading raw float32 operands as
    tf32 takes their top 19 bits)."""
    u = np.asarray(x, f32).view(np.uint32).astype(np.uint64)
    u = ((u if trunc else u + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return u.view(f32).astype(np.float64)


def bf16_bits_rn(x):
    """float32 -> bf16 bit patterns, round to nearest even."""
    u = np.asarray(x, f32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


# --------------------------------------------------------------------------
# the reference's open problems (problems/*/meta.json "code")
# --------------------------------------------------------------------------

def _const(v, name):
    return float(np.asarray(v[name]).reshape(-1)[0])


PROBLEMS = {
    "p00_scalar_add": lambda v: {"add": add_f32(v["x0"], v["x1"])},
    "p01_vector_add": lambda v: {"add": add_f32(v["x0"], v["x1"])},
    "p02_scale_shift": lambda v: {"add": scale_shift_f32(v["x"], _const(v, "mul_c1"),
                                                         _const(v, "add_c1"))},
    "p03_relu_mul": lambda v: {"mul": relu_mul_f32(v["x"], v["y"])},
    "r01_array_sum": lambda v: {"sum_1": full_sum(v["x"])},
    "r02_big_sum": lambda v: {"sum_1": full_sum(v["x"])},
    "r03_mean": lambda v: {"mean": full_mean(v["x"])},
    "r04_row_sum": lambda v: {"sum_1": row_sum(v["x"])},
    "f01_rmsnorm": lambda v: {"mul_1": rmsnorm(v["x"], v["w"], _const(v, "add_c1"))},
    "f02_row_softmax": lambda v: {"softmax": softmax_rows(v["x"])},
    "f03_l2norm": lambda v: {"div": l2norm(v["x"])},
    "m01_matmul_512": lambda v: {"matmul": matmul(v["x0"], v["x1"])},
    "m02_matmul_rect": lambda v: {"matmul": matmul(v["x0"], v["x1"])},
    "a01_attention": lambda v: {"matmul_1": attention(v["q"], v["kt"], v["v"],
                                                      1.0 / _const(v, "div_c1"), True)},
    "a02_attention_128": lambda v: {"matmul_1": attention(v["q"], v["kt"], v["v"],
                                                          1.0 / _const(v, "div_c1"), True)},
}


def evaluate_problem(problem_id: str, inputs: dict) -> dict:
    return PROBLEMS[problem_id](inputs)


# --------------------------------------------------------------------------
# synthesised configurations: the IR synthesiser records {"family", params}
# in meta["oracle"]; inputs are keyed by buffer name
# --------------------------------------------------------------------------

def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def evaluate_family(spec: dict, inputs: dict) -> dict:
    fam = spec["family"]
    a = spec.get("args", {})
    v = {k: (bf16_to_f32(x) if spec.get("bf16", {}).get(k) else x) for k, x in inputs.items()}
    out = spec["output"]
    if fam == "add":
        r = add_f32(v[a["a"]], v[a["b"]])
    elif fam == "sum":
        r = full_sum(v[a["x"]])
    elif fam == "row_sum":
        r = row_sum(v[a["x"]])
    elif fam == "row_mean":
        r = row_mean(v[a["x"]])
    elif fam == "rmsnorm":
        r = rmsnorm(v[a["x"]], v[a["w"]], spec["eps"])
    elif fam == "softmax":
        r = softmax_rows(v[a["x"]], spec.get("scale", 1.0))
    elif fam == "l2norm":
        r = l2norm(v[a["x"]], spec.get("eps"))
    elif fam == "matmul":
        r = matmul(v[a["a"]], v[a["b"]])
    elif fam == "attention":
        r = attention(v[a["q"]], v[a["k"]], v[a["v"]], spec["scale"])
    elif fam == "carried_prefix":
        r = carried_prefix(v[a["x"]], spec["every"])
    elif fam == "select":
        r = select_split(v[a["x"]], spec["split"])
    elif fam == "zero_prologue":
        r = zero_prologue(v[a["x"]], spec["words"])
    elif fam == "mma_matmul":
        r = mma_matmul(v[a["a"]], v[a["b"]], spec["b_kn"],
                       v.get(a["bias"]) if spec.get("epilogue") else None,
                       spec.get("tf32", False), spec.get("out_bf16", False))
    elif fam == "mma_attention":
        r = mma_attention(v[a["q"]], v[a["k"]], v[a["v"]], spec["scale"], spec.get("causal"),
                          v.get(a["bias"]) if spec.get("bias_on") else None)
    else:
        raise KeyError(fam)
    return {out: r}


def tolerance(spec_or_meta: dict, ref: np.ndarray) -> tuple[float, float]:
    """(rtol, atol): the problem's own pair, with atol = rtol * max|ref| when the
    problem gives none (the survey's recommendation for non-pointwise checks)."""
    rtol = float(spec_or_meta.get("rtol", 0.0))
    atol = spec_or_meta.get("atol")
    if atol is None:
        atol = rtol * float(np.max(np.abs(ref))) if ref.size else 0.0
    return rtol, float(atol)

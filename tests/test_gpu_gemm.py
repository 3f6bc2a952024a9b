"""Parity on the GPU for the tcgen05 matmul template (bf16 inputs, f32
accumulate) against the float64 CPU oracle on the same bf16-rounded inputs,
rel 2e-2 with atol = rtol * max|ref|: small and tile-edge shapes in full, the
BASELINE shape (M=16384, N=8192, K=4096) on sampled rows.  The kernel's
bounded waits must not have fired (module status word stays 0)."""
import numpy as np
import pytest

from emmy_b200 import synth
from emmy_b200.data import bf16_to_f32, materialize
from oracle import expr

pytestmark = pytest.mark.gpu

CASES = [
    dict(M=128, N=256, K=64),                    # one tile, one k-step
    dict(M=256, N=256, K=128),
    dict(M=512, N=512, K=1024),                  # ring wraps (16 k-steps, 4 stages)
    dict(M=256, N=256, K=256, BN=128, U0=8, U1=32),
    dict(M=256, N=512, K=192, BN=64, U0=16, U1=16, BK=64),
]


def _run(p, rows=None):
    from emmy_b200 import harness
    g, m = p.build()
    k = m["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    outs, kern = harness.run(g, m, ins)
    assert kern.kind == "gemm"
    addr, n = kern.module().global_addr("__emmy_status")
    import ctypes
    import torch
    st = torch.zeros(1, dtype=torch.int32)
    from emmy_b200 import native
    native.check(native.lib().emmy_memcpy_dtoh_async(st.data_ptr(), addr, 4, None))
    torch.cuda.synchronize()
    assert int(st[0]) == 0, f"bounded wait fired, status {int(st[0])}"
    a = ins["x0"] if rows is None else ins["x0"][rows]
    ref = expr.evaluate_family(m["oracle"], {"x0": a, "x1": ins["x1"]})["matmul"]
    got = outs["matmul"] if rows is None else outs["matmul"][rows]
    rtol, atol = expr.tolerance(m, ref)
    err = np.max(np.abs(got - ref))
    assert np.allclose(got, ref, rtol=rtol, atol=atol), err
    return got, ref


@pytest.mark.parametrize("kw", CASES, ids=[f"{c['M']}x{c['N']}x{c['K']}" for c in CASES])
def test_gemm_small(kw):
    got, ref = _run(synth.matmul(**kw))
    # bf16 products accumulate exactly enough in f32 that the error is tiny
    assert np.max(np.abs(got - ref)) <= 1e-3 * max(1.0, float(np.max(np.abs(ref))))


def test_gemm_baseline_rows():
    """BASELINE shape, 2-stage IR ring: the per-tile CTA-pair kernel."""
    p = synth.matmul()
    rows = np.sort(np.random.default_rng(3).choice(16384, 48, replace=False))
    _run(p, rows=rows)


def test_gemm_baseline_rows_persistent():
    """BASELINE shape as benchmarked (4-stage IR ring): the persistent
    CTA-pair kernel, 28 tiles per worker cluster."""
    p = synth.config("matmul_bf16")
    rows = np.sort(np.random.default_rng(11).choice(16384, 48, replace=False))
    _run(p, rows=rows)


F32_CASES = [dict(M=128, N=256, K=32), dict(M=256, N=256, K=128), dict(M=512, N=512, K=1024),
             dict(M=256, N=256, K=256, BN=128, U0=8, U1=32)]


@pytest.mark.parametrize("kw", F32_CASES, ids=[f"{c['M']}x{c['N']}x{c['K']}" for c in F32_CASES])
def test_gemm_f32_3xtf32(kw):
    """fp32 inputs through the 3xTF32 split: rel 1e-4 (BASELINE), and in
    practice close to fp32 accuracy (checked at 2e-5 of max|C|)."""
    got, ref = _run(synth.config("matmul_f32", **kw))
    assert np.max(np.abs(got - ref)) <= 2e-5 * max(1.0, float(np.max(np.abs(ref))))


def test_gemm_f32_baseline_rows():
    p = synth.config("matmul_f32")
    rows = np.sort(np.random.default_rng(4).choice(16384, 32, replace=False))
    _run(p, rows=rows)


PAIR_CASES = [dict(M=256, N=256, K=64), dict(M=256, N=256, K=128),
              dict(M=1024, N=768, K=512), dict(M=512, N=512, K=1024)]


@pytest.mark.parametrize("pair", [True, False], ids=["pair", "single"])
@pytest.mark.parametrize("kw", PAIR_CASES, ids=[f"{c['M']}x{c['N']}x{c['K']}" for c in PAIR_CASES])
def test_gemm_pair_and_single(kw, pair, monkeypatch):
    """bf16 128x256 tiles run on CTA pairs (cta_group::2) by default; the
    same shapes through the single-CTA kernel must agree with the oracle
    too, so both code paths stay covered."""
    from emmy_b200.templates import gemm
    monkeypatch.setattr(gemm.GemmTemplate, "PAIR", pair)
    from emmy_b200 import compiler
    g, m = synth.matmul(**kw).build()
    assert ("cta_group::2" in compiler.compile_graph(g, m).render()) == pair
    got, ref = _run(synth.matmul(**kw))
    assert np.max(np.abs(got - ref)) <= 1e-3 * max(1.0, float(np.max(np.abs(ref))))


PERSISTENT_CASES = [dict(M=256, N=256, K=64), dict(M=1024, N=768, K=512),
                    dict(M=512, N=512, K=1024), dict(M=4096, N=2048, K=512),
                    dict(M=8192, N=4096, K=256), dict(M=2048, N=8192, K=256),
                    dict(M=1024, N=5120, K=256)]


@pytest.mark.parametrize("kw", PERSISTENT_CASES,
                         ids=[f"{c['M']}x{c['N']}x{c['K']}" for c in PERSISTENT_CASES])
def test_gemm_persistent_pairs(kw):
    """IR rings of 4 stages (198 KiB: one CTA per SM) run the persistent
    pair kernel: 74 worker clusters, two tensor-memory accumulators, the
    epilogue of tile i overlapping the main loop of tile i+1.  The large
    shapes give each worker up to 7 tiles (both accumulators reused several
    times) and are checked on sampled rows; 2048 x 8192 (256 tiles: 3 full
    rounds, 34 leftover tiles as 68 halves of 256 x 128) and 1024 x 5120
    (80 tiles: 6 leftover as 12 halves) run the split tail."""
    from emmy_b200 import compiler
    p = synth.matmul(stages=4, **kw)
    g, m = p.build()
    assert "persistent CTA pairs" in compiler.compile_graph(g, m).render()
    rows = None
    if kw["M"] >= 4096:
        rows = np.sort(np.random.default_rng(7).choice(kw["M"], 64, replace=False))
    got, ref = _run(p, rows=rows)
    assert np.max(np.abs(got - ref)) <= 1e-3 * max(1.0, float(np.max(np.abs(ref))))


F32_PERSISTENT_CASES = [dict(M=256, N=256, K=128), dict(M=1024, N=768, K=256),
                        dict(M=4096, N=2048, K=256), dict(M=8192, N=4096, K=128),
                        dict(M=2048, N=8192, K=128), dict(M=1024, N=5120, K=128)]


@pytest.mark.parametrize("kw", F32_PERSISTENT_CASES,
                         ids=[f"{c['M']}x{c['N']}x{c['K']}" for c in F32_PERSISTENT_CASES])
def test_gemm_f32_persistent_pairs(kw, monkeypatch):
    """fp32 operands on persistent CTA pairs with both operands in shared
    memory (``TF32_A_TMEM`` off): each CTA's converter warps write the tf32
    low parts of its landed slice and arrive on the leader's conversion
    barrier; the leader issues lo*hi, hi*lo, hi*hi as ``kind::tf32`` pair
    MMAs; warps 4-7 drain the previous tile's accumulator.  Rel 2e-5 of
    max|C| (BASELINE asks 1e-4); large shapes on sampled rows; the last two
    shapes run the split 256 x 128 tail."""
    from emmy_b200 import compiler
    from emmy_b200.templates import gemm_persistent
    monkeypatch.setattr(gemm_persistent, "TF32_A_TMEM", False)
    p = synth.config("matmul_f32", **kw)
    g, m = p.build()
    assert "persistent CTA pairs" in compiler.compile_graph(g, m).render()
    rows = None
    if kw["M"] >= 4096:
        rows = np.sort(np.random.default_rng(9).choice(kw["M"], 64, replace=False))
    got, ref = _run(p, rows=rows)
    assert np.max(np.abs(got - ref)) <= 2e-5 * max(1.0, float(np.max(np.abs(ref))))


def test_gemm_f32_3xtf32_error_against_float64():
    """3xTF32 with the raw fp32 slice as the high part: the normwise error
    against float64 at 1024 x 1024 x 4096 stays inside the fp32 matmul's rel
    1e-4 (measured 2.9e-5, the same as with rounded high parts) and the mean
    error shows no offset.  A tensor core that rounded the raw element to tf32
    instead of dropping its 13 low bits would leave lo = x - trunc(x) off by up
    to a tf32 ulp per element, a normwise error near 2^-12, which the first
    bound rejects."""
    from emmy_b200 import harness
    p = synth.matmul(dtype="f32", BK=32, stages=4, M=1024, N=1024, K=4096)
    g, m = p.build()
    k = m["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    outs, kern = harness.run(g, m, ins)
    assert kern.kind == "gemm"
    A = ins["x0"].astype(np.float64).reshape(1024, 4096)
    B = ins["x1"].astype(np.float64).reshape(4096, 1024)
    ref = A @ B
    got = outs["matmul"].astype(np.float64).reshape(1024, 1024)
    nrm = np.linalg.norm(ref)
    assert np.linalg.norm(got - ref) / nrm < 1e-4
    assert abs(float((got - ref).mean())) * 1024 / nrm < 1e-6


@pytest.mark.parametrize("kw", F32_PERSISTENT_CASES,
                         ids=[f"{c['M']}x{c['N']}x{c['K']}" for c in F32_PERSISTENT_CASES])
def test_gemm_f32_persistent_pairs_a_in_tmem(kw, monkeypatch):
    """3xTF32 with the A operand in tensor memory (``TF32_A_TMEM``, the
    default, set here explicitly): warps
    4-7 store each A row's raw values and low parts into the stage's TMEM
    columns, the MMAs read A there (``[a-tmem]``) and B from shared memory,
    one accumulator (each tile drained before the next one's MMAs).  The
    same bounds as the shared-memory form."""
    from emmy_b200 import compiler
    from emmy_b200.templates import gemm_persistent
    monkeypatch.setattr(gemm_persistent, "TF32_A_TMEM", True)
    p = synth.config("matmul_f32", **kw)
    g, m = p.build()
    ptx = compiler.compile_graph(g, m).render()
    import re
    assert "persistent CTA pairs" in ptx
    assert re.search(r"kind::tf32 \[%r\d+\], \[%r\d+\]", ptx)     # A from tensor memory
    rows = None
    if kw["M"] >= 4096:
        rows = np.sort(np.random.default_rng(9).choice(kw["M"], 64, replace=False))
    got, ref = _run(p, rows=rows)
    assert np.max(np.abs(got - ref)) <= 2e-5 * max(1.0, float(np.max(np.abs(ref))))

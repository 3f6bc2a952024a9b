"""The tcgen05 kernels with a meta-only launch (``templates/gemm_small.py``,
``templates/attention_small.py``) on the GPU: Emmy's own matmul and attention
IRs (the a01/a02 open problems and the corpus attn* IRs, fp32 with K
pre-transposed, one-row to 32-row CTA blocks, grouped rasterisation) and matmul IRs (the m01/m02 open problems, the corpus mm*
IRs: odd CTA tiles, edge guards, split K with atomic stores) against their
golden outputs; the same kernels launched by a bare CUDA-driver launcher that
passes exactly the meta ``arg_order`` (``cuModuleLoadData`` on the PTX text,
``cuLaunchKernel``, as the reference's ``tools/harness/gpu_run.py:46-103``
does); and, with ``EMMY_META_ONLY=1``, the synthesised benchmark matmuls
(fp32 through 3xTF32, bf16) against the float64 oracle.  The kernel's bounded
waits must not have fired (status word 0)."""
import ctypes
import json

import numpy as np
import pytest

from conftest import GOLDEN
from emmy_b200 import synth
from emmy_b200.data import materialize
from oracle import expr

pytestmark = pytest.mark.gpu

EMMY_MATMULS = [GOLDEN / "problems" / "m01_matmul_512", GOLDEN / "problems" / "m02_matmul_rect"] + \
    [GOLDEN / "corpus" / n for n in ("mm128", "mm256", "mm512", "mm64a", "mm_rect2")]
EMMY_ATTENTION = [GOLDEN / "problems" / "a01_attention", GOLDEN / "problems" / "a02_attention_128"] + \
    [GOLDEN / "corpus" / n for n in ("attn128b", "attn64b", "attn96")]


def _status(kern):
    import torch
    from emmy_b200 import native
    addr, _ = kern.module().global_addr("__emmy_status")
    st = torch.zeros(1, dtype=torch.int32)
    native.check(native.lib().emmy_memcpy_dtoh_async(st.data_ptr(), addr, 4, None))
    torch.cuda.synchronize()
    return int(st[0])


@pytest.mark.parametrize("folder", EMMY_MATMULS, ids=lambda p: p.name)
def test_emmy_matmul_irs_on_tensor_cores(folder, monkeypatch):
    from emmy_b200 import harness
    from emmy_b200.templates.gemm_small import GemmSmallTemplate
    # the tcgen05 form also for the IRs whose little work a thread the
    # selection sends to the generic lowering
    monkeypatch.setattr(GemmSmallTemplate, "MIN_MACS_PER_THREAD", 0)
    g = json.loads((folder / "kernel.ir.json").read_text())
    meta = json.loads((folder / "meta.json").read_text())
    outs, kern = harness.run(g, meta, folder=folder)
    assert kern.kind == "gemm" and type(kern.compiler.template).__name__ == "GemmSmallTemplate"
    assert not kern.tmaps
    assert _status(kern) == 0
    _check_expected(folder, meta, outs)


@pytest.mark.parametrize("folder", EMMY_ATTENTION, ids=lambda p: p.name)
def test_emmy_attention_irs_on_tensor_cores(folder):
    from emmy_b200 import harness
    g = json.loads((folder / "kernel.ir.json").read_text())
    meta = json.loads((folder / "meta.json").read_text())
    outs, kern = harness.run(g, meta, folder=folder)
    assert kern.kind == "attention" and \
        type(kern.compiler.template).__name__ == "AttentionSmallTemplate"
    assert not kern.tmaps
    assert _status(kern) == 0
    _check_expected(folder, meta, outs)


def _check_expected(folder, meta, outs):
    """Golden outputs: an open problem's expected.npz is keyed by output name;
    a corpus case's holds ``val`` (and ``idx`` when sampled)."""
    exp = np.load(folder / "expected.npz")
    out = next(a for a in meta["kernels"][0]["args"] if a.get("output"))["name"]
    got = np.asarray(outs[out]).astype(np.float64).reshape(-1)
    if "val" in exp:
        ref = exp["val"].astype(np.float64).reshape(-1)
        if "idx" in exp:
            got = got[exp["idx"]]
    else:
        ref = exp[out].astype(np.float64).reshape(-1)
    assert got.shape == ref.shape
    assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]), \
        float(np.max(np.abs(got - ref)))


@pytest.mark.parametrize("folder", EMMY_MATMULS[:3] + EMMY_ATTENTION[:2], ids=lambda p: p.name)
def test_bare_driver_launch_with_meta_arguments(folder):
    """Load the PTX text with the CUDA driver and launch it with exactly the
    meta arguments: no tensor maps, no library of this build in the launch."""
    import torch
    from cuda.bindings import driver as cu
    from emmy_b200.compiler import compile_graph
    g = json.loads((folder / "kernel.ir.json").read_text())
    meta = json.loads((folder / "meta.json").read_text())
    kinfo = meta["kernels"][0]
    ptx = compile_graph(g, meta).render()
    assert "@emmy tmap" not in ptx
    torch.cuda.init()
    torch.zeros(1, device="cuda")                       # the primary context, current
    err, mod = cu.cuModuleLoadData(ptx.encode() + b"\0")
    assert err == cu.CUresult.CUDA_SUCCESS, err
    err, fn = cu.cuModuleGetFunction(mod, kinfo["entry"].encode())
    assert err == cu.CUresult.CUDA_SUCCESS, err
    if kinfo["smem_bytes"] > 48 * 1024:
        (err,) = cu.cuFuncSetAttribute(
            fn, cu.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
            kinfo["smem_bytes"])
        assert err == cu.CUresult.CUDA_SUCCESS, err
    bufs, vals = {}, []
    for a in kinfo["args"]:
        if a.get("output"):
            bufs[a["name"]] = torch.zeros(int(np.prod(a["shape"])), dtype=torch.float32,
                                          device="cuda")
        else:
            bufs[a["name"]] = torch.from_numpy(materialize(a, folder).reshape(-1)).cuda()
    keep = [ctypes.c_uint64(bufs[n].data_ptr()) for n in kinfo["arg_order"]]
    params = (ctypes.c_void_p * len(keep))(*[ctypes.addressof(v) for v in keep])
    (err,) = cu.cuLaunchKernel(fn, *kinfo["grid"], *kinfo["block"], kinfo["smem_bytes"], 0,
                               ctypes.addressof(params), 0)
    assert err == cu.CUresult.CUDA_SUCCESS, err
    torch.cuda.synchronize()
    _check_expected(folder, meta, {n: t.cpu().numpy() for n, t in bufs.items()})
    cu.cuModuleUnload(mod)


META_CASES = [dict(M=256, N=256, K=128, dtype="f32", BK=32),
              dict(M=512, N=512, K=1024, dtype="f32", BK=32, stages=4),
              dict(M=256, N=512, K=256, dtype="bf16"),
              dict(M=512, N=256, K=512, dtype="bf16", stages=4)]


@pytest.mark.parametrize("kw", META_CASES, ids=[f"{c['dtype']}_{c['M']}x{c['N']}x{c['K']}"
                                                for c in META_CASES])
def test_meta_only_benchmark_form(kw, monkeypatch):
    """EMMY_META_ONLY=1: the benchmark's matmul IRs (128 x 256 CTA tiles, 256
    threads) on the meta-only kernel; fp32 within 2e-5 of max|C| (3xTF32),
    bf16 within 1e-3."""
    from emmy_b200 import harness
    monkeypatch.setenv("EMMY_META_ONLY", "1")
    g, m = synth.matmul(**kw).build()
    k = m["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    outs, kern = harness.run(g, m, ins)
    assert type(kern.compiler.template).__name__ == "GemmSmallTemplate" and not kern.tmaps
    assert _status(kern) == 0
    ref = expr.evaluate_family(m["oracle"], ins)["matmul"]
    got = outs["matmul"]
    bound = 2e-5 if kw["dtype"] == "f32" else 1e-3
    assert np.max(np.abs(got - ref)) <= bound * max(1.0, float(np.max(np.abs(ref))))


@pytest.mark.parametrize("name", ["matmul_bf16", "matmul_f32"])
def test_meta_only_baseline_rows(name, monkeypatch):
    """The BASELINE shape (16384 x 8192 x 4096) on the meta-only kernel,
    sampled rows against the float64 oracle at the BASELINE tolerances."""
    from emmy_b200 import harness
    monkeypatch.setenv("EMMY_META_ONLY", "1")
    p = synth.config(name)
    g, m = p.build()
    k = m["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    outs, kern = harness.run(g, m, ins)
    assert type(kern.compiler.template).__name__ == "GemmSmallTemplate"
    assert _status(kern) == 0
    rows = np.sort(np.random.default_rng(13).choice(16384, 16, replace=False))
    ref = expr.evaluate_family(m["oracle"], {"x0": ins["x0"][rows], "x1": ins["x1"]})["matmul"]
    got = outs["matmul"][rows]
    rtol, atol = expr.tolerance(m, ref)
    assert np.allclose(got, ref, rtol=rtol, atol=atol), float(np.max(np.abs(got - ref)))

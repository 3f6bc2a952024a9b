"""The register-fragment tensor-core statements (``mma.sync``; reference
TASK.md "Tensor core: register fragments", rows marked * -- defined by the
vocabulary, used by no reference IR, exit 1 in the reference compiler)
lowered by ``emmy_b200.fragments`` on sm_100a, run on IRs written in the
forms that module documents (``synth.mma_matmul``, ``synth.mma_attention``)
and checked against the oracle restated from the same descriptions
(``oracle.expr.mma_matmul`` / ``mma_attention``)."""
import numpy as np
import pytest

from emmy_b200 import synth
from emmy_b200.data import materialize
from oracle import expr

pytestmark = pytest.mark.gpu


def _run(p):
    from emmy_b200 import harness
    g, m = p.build()
    kern = harness.CompiledKernel(g, m)
    assert kern.kind == "generic"
    k = m["kernels"][0]
    ins = {a["name"]: materialize(a) for a in k["args"] if not a.get("output")}
    outs, _ = harness.run(g, m, ins, kern=kern)
    spec = m["oracle"]
    ref = expr.evaluate_family(spec, ins)[spec["output"]]
    got = outs[spec["output"]]
    if k["args"][-1]["dtype"] == "bf16":
        got = expr.bf16_to_f32(got)
    got = np.asarray(got, np.float32).reshape(ref.shape)
    rtol, atol = expr.tolerance(m, ref)
    assert np.all(np.isfinite(got))
    assert np.allclose(got, ref, rtol=rtol, atol=atol), float(np.max(np.abs(got - ref)))


@pytest.mark.parametrize("kw", [
    dict(), dict(b_kn=False), dict(stage=False), dict(stage=False, b_kn=False),
    dict(M=256, N=192, K=128), dict(M=1, N=5, K=7, stage=False),
    dict(dtype="f16"), dict(dtype="f16", promote=True),
    dict(dtype="tf32"), dict(dtype="tf32", stage=False, b_kn=False),
    dict(epilogue=True), dict(epilogue=True, out_dtype="bf16"), dict(split_k=3, K=200),
    dict(swizzle=True), dict(swizzle=True, b_kn=False, K=200)],
    ids=["smem", "smem_nk", "direct", "direct_nk", "aligned", "tiny", "f16", "f16_promote",
         "tf32", "tf32_direct_nk", "epilogue", "epilogue_bf16", "split_k", "swizzled",
         "swizzled_nk"])
def test_mma_matmul(kw):
    """ldmatrix (plain and .trans, unswizzled and through the 128-byte chunk
    swizzle) and guarded element loads, bf16 / f16 /
    tf32 mma.sync, f16 accumulators promoted into f32, the store's Lambda
    epilogue, bf16 stores, atomic split-K stores; ragged 200 x 136 x 80 by
    default (edge tiles cut by the guards)."""
    _run(synth.mma_matmul(**kw))


@pytest.mark.parametrize("kw", [dict(), dict(causal=True), dict(bias=True),
                                dict(Sq=100, Sk=128, d=64, causal=True, bias=True)],
                         ids=["plain", "causal", "bias", "ragged_all"])
def test_mma_attention(kw):
    """Row max / sum by FragmentRowReduce, scale, mask and bias arguments of
    FragmentApply, exp2 as its post op, P repacked to bf16 A fragments, O / l
    by a row argument, guarded stores of a ragged last query block."""
    _run(synth.mma_attention(**kw))


@pytest.mark.parametrize("kw", [dict(), dict(layout="sw128_mn", BN=128), dict(layout="none"),
                                dict(pipelined=True), dict(warpgroups=2, BN=128),
                                dict(dtype="f16", M=128, N=64, K=64), dict(a_regs=True),
                                dict(a_regs=True, warpgroups=2, BN=128, layout="sw128_mn"),
                                dict(dtype="tf32"), dict(dtype="tf32", layout="none")],
                         ids=["sw128", "sw128_mn", "no_swizzle", "pipelined", "two_warpgroups",
                              "f16_aligned", "a_in_registers", "a_in_registers_wg2_mn",
                              "tf32_sw128", "tf32_no_swizzle"])
def test_wgmma_matmul(kw):
    """The warpgroup statements on tcgen05: M = 64 accumulators in tensor
    memory read back into the warps' C fragments, K-major and MN-major
    128-byte-swizzled and unswizzled descriptors, a commit per slab with
    WgmmaWait(1) over two slab buffers, two warpgroups a CTA (their own
    accumulator columns and barriers), the A operand from registers (staged
    through the unswizzled K-major slot), tf32 operands (m64nNk8: raw float32
    read as tf32, against an oracle that truncates them the same way),
    ragged 200 x 136 x 200 by default."""
    _run(synth.wgmma_matmul(**kw))

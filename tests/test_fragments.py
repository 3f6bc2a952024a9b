"""CPU checks of the register-fragment statements: every synthesised IR
compiles through the generic lowering, assembles for sm_100a and passes
the static checkers; the forms sm_100a cannot run exit 1."""
import json
import shutil
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from emmy_b200 import ir as I
from emmy_b200 import ptxcheck, synth
from emmy_b200.compiler import compile_graph
from oracle import expr

REPO = Path(__file__).resolve().parents[1]

CASES = {
    "smem": dict(), "smem_nk": dict(b_kn=False), "direct": dict(stage=False),
    "f16_promote": dict(dtype="f16", promote=True), "tf32": dict(dtype="tf32"),
    "epilogue_bf16": dict(epilogue=True, out_dtype="bf16"), "split_k": dict(split_k=3, K=200),
    "swizzled": dict(swizzle=True),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_mma_matmul_compiles(name):
    g, m = synth.mma_matmul(**CASES[name]).build()
    c = compile_graph(g, m)
    assert c.kind == "generic"
    assert "mma.sync.aligned" in c.ptx
    assert ptxcheck.check(c.ptx) == []
    if shutil.which("ptxas"):
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", "-"],
                           input=c.ptx, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_mma_attention_compiles():
    g, m = synth.mma_attention(Sq=100, causal=True, bias=True).build()
    c = compile_graph(g, m)
    for ins in ("ldmatrix.sync.aligned.m8n8.x2.trans", "shfl.sync.bfly",
                "cvt.rn.bf16x2.f32", "mma.sync.aligned.m16n8k16"):
        assert ins in c.ptx
    assert ptxcheck.check(c.ptx) == []


def test_round_trip_repr():
    """The fragment statements serialise and parse back unchanged."""
    p = synth.mma_attention(causal=True, bias=True)
    body = p.graph()["nodes"]["o"]["op_fields"]["body"][0]
    assert I.parse_repr(body) == p.body


def _cli(tmp_path, g, m):
    (tmp_path / "k.ir.json").write_text(json.dumps(g))
    (tmp_path / "meta.json").write_text(json.dumps(m))
    return subprocess.run([sys.executable, str(REPO / "compile.py"), str(tmp_path / "k.ir.json")],
                          capture_output=True, text=True)


def test_block_scaled_is_exit_1(tmp_path):
    """Block-scaled mma.sync is an sm_120a instruction: exit 1, unsupported."""
    g, m = synth.mma_matmul().build()
    body = g["nodes"]["c"]["op_fields"]["body"][0]
    g["nodes"]["c"]["op_fields"]["body"][0] = body.replace(
        "sfa_frag=None", "sfa_frag='fa[0]'", 1)
    r = _cli(tmp_path, g, m)
    assert r.returncode == 1 and r.stderr.startswith("unsupported construct:")
    assert "sm_120a" in r.stderr


def test_oracle_tf32_rounding():
    """cvt.rna.tf32.f32: 10 mantissa bits kept, ties away from zero."""
    x = np.array([1.0, 1.0 + 2 ** -11, 1.0 + 2 ** -10 + 2 ** -11, -(1.0 + 2 ** -11)], np.float32)
    assert list(expr._tf32(x)) == [1.0, 1.0 + 2 ** -10, 1.0 + 2 ** -9, -(1.0 + 2 ** -10)]


@pytest.mark.parametrize("kw", [dict(), dict(layout="sw128_mn", BN=128), dict(layout="none"),
                                dict(pipelined=True), dict(warpgroups=2, BN=128),
                                dict(a_regs=True)],
                         ids=["sw128", "sw128_mn", "none", "pipelined", "wg2", "a_regs"])
def test_wgmma_compiles(kw):
    """wgmma on sm_100a: tcgen05.mma M = 64 into tensor memory, 16x256b
    loads and stores of the C fragments, TMEM freed at the end; the static
    checkers pass (TMEM pairing, bounded mbarrier waits, definedness)."""
    g, m = synth.wgmma_matmul(**kw).build()
    c = compile_graph(g, m)
    assert c.kind == "generic"
    for ins in ("tcgen05.mma.cta_group::1.kind::f16", "tcgen05.ld.sync.aligned.16x256b",
                "tcgen05.st.sync.aligned.16x256b", "tcgen05.dealloc", "fence.proxy.async"):
        assert ins in c.ptx
    assert ptxcheck.check(c.ptx) == []
    if shutil.which("ptxas"):
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", "-"],
                           input=c.ptx, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_wgmma_tf32_register_a_is_exit_1(tmp_path):
    """A register A operand of tf32 has no staged form here: exit 1."""
    g, m = synth.wgmma_matmul(a_regs=True).build()
    body = g["nodes"]["c"]["op_fields"]["body"][0]
    g["nodes"]["c"]["op_fields"]["body"][0] = body.replace("m64n64k16", "m64n64k8")
    r = _cli(tmp_path, g, m)
    assert r.returncode == 1 and r.stderr.startswith("unsupported construct:")


@pytest.mark.parametrize("role,kk,cls,rows,cols", [
    ("a", 16, "wide", 16, 16), ("a", 8, "wide", 16, 8), ("a", 8, "tf32", 16, 8),
    ("b", 16, "wide", 16, 8), ("b", 8, "wide", 8, 8), ("b", 8, "tf32", 8, 8),
    ("c", 16, "f32", 16, 8), ("c", 16, "f16", 16, 8)])
def test_fragment_layouts_cover_the_tile_once(role, kk, cls, rows, cols):
    """Every element of an operand tile (A m x k, B k x n, C m x n) is held by
    exactly one (lane, register, half) of the warp under the mma.sync layouts
    the fragment statements use."""
    from emmy_b200.fragments import _LAYOUTS
    lay = _LAYOUTS[(role, kk, cls)]
    seen = {}
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        for (reg, half, r, c) in lay:
            row = r[0] * g + r[1] * t + r[2]
            col = c[0] * g + c[1] * t + c[2]
            assert 0 <= row < rows and 0 <= col < cols
            assert (row, col) not in seen, ((row, col), seen.get((row, col)), (lane, reg, half))
            seen[(row, col)] = (lane, reg, half)
    assert len(seen) == rows * cols


def _body_edit(g, old, new):
    node = next(n for n in g["nodes"].values() if n["op"] == "KernelOp")
    body = node["op_fields"]["body"][0]
    assert old in body, old
    node["op_fields"]["body"][0] = body.replace(old, new, 1)


@pytest.mark.parametrize("old,new,msg", [
    ("RegFragment(name='fa', role='a', shape='m16n8k16'",
     "RegFragment(name='fa', role='a', shape='m16n8k32'", "shape"),
    ("count=2, nregs=4)", "count=2, nregs=3)", "registers"),
    ("MmaSyncPtx(c_frag='acc[0]', a_frag='fa[0]', b_frag='fb[0]'",
     "MmaSyncPtx(c_frag='acc[0]', a_frag='fb[0]', b_frag='fa[0]'", "operands"),
    ("LdmatrixLoad(frag='fa[0]'", "LdmatrixLoad(frag='nope[0]'", "before its RegFragment"),
    ("volta_interleaved=False", "volta_interleaved=True", "volta_interleaved"),
], ids=["shape", "nregs", "roles", "undeclared", "volta"])
def test_fragment_misuse_is_exit_1(tmp_path, old, new, msg):
    """Fragment statements this lowering cannot honour -- an mma shape it
    has no layout for, a register count that contradicts the shape, A and B
    swapped, a fragment used before its declaration, Volta-interleaved
    stores -- exit 1 with ``unsupported construct`` and the reason."""
    g, m = synth.mma_matmul().build()
    _body_edit(g, old, new)
    r = _cli(tmp_path, g, m)
    assert r.returncode == 1 and r.stderr.startswith("unsupported construct:"), r.stderr
    assert msg in r.stderr, r.stderr

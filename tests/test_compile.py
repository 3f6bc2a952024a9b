"""compile.py contract (reference compile.py:2651-2668, TASK.md:1-33) and
that every emitted kernel assembles for sm_100a (in-process ptxas through
the C-ABI library; no GPU needed)."""
import json
import re
import shutil
import subprocess
import sys

import pytest

from conftest import PROBLEMS, REPO

from emmy_b200 import synth
from emmy_b200.compiler import compile_graph

TEMPLATED = {"p00_scalar_add": "pointwise", "p01_vector_add": "pointwise",
             "p02_scale_shift": "pointwise", "p03_relu_mul": "pointwise",
             "r01_array_sum": "rows", "r02_big_sum": "rows", "r03_mean": "rows",
             "r04_row_sum": "rows", "f01_rmsnorm": "rows", "f02_row_softmax": "rows",
             "f03_l2norm": "rows"}

CONFIGS = ["vector_add", "full_sum", "row_sum", "row_mean", "rmsnorm", "softmax", "l2norm"]


def _cli(*args, cwd=None):
    return subprocess.run([sys.executable, str(REPO / "compile.py"), *args],
                          capture_output=True, text=True, cwd=cwd)


@pytest.mark.parametrize("pid", sorted(TEMPLATED))
def test_cli_emits_sm100a(pid, native_lib):
    from emmy_b200 import native
    r = _cli(str(REPO / "tests/golden/problems" / pid / "kernel.ir.json"))
    assert r.returncode == 0, r.stderr
    ptx = r.stdout
    assert ptx.startswith(".version 8.8\n.target sm_100a\n.address_size 64\n")
    assert ptx.isascii()
    meta = json.loads((REPO / "tests/golden/problems" / pid / "meta.json").read_text())
    k = meta["kernels"][0]
    # entry = KernelOp name, params = meta arg_order
    m = re.search(r"\.visible \.entry (\w+)\(([^)]*)\)", ptx)
    assert m and m.group(1) == k["entry"]
    params = re.findall(r"param_(\w+)", m.group(2))
    assert params == k["arg_order"]
    img = native.Image(ptx)
    assert len(img.data) > 0 and k["entry"] in img.registers()


def test_cli_usage_and_missing_meta(tmp_path):
    assert _cli().returncode == 2
    src = REPO / "tests/golden/problems/p01_vector_add/kernel.ir.json"
    shutil.copy(src, tmp_path / "k.ir.json")
    r = _cli(str(tmp_path / "k.ir.json"))
    assert r.returncode == 2 and "meta.json" in r.stderr


def test_cli_unsupported_is_exit_1(tmp_path):
    # a statement sm_100a cannot lower (block-scaled mma.sync is sm_120a-only)
    # -> exit 1, "unsupported construct"
    g, m = synth.vector_add(n=1024, threads=256).build()
    body = g["nodes"]["add"]["op_fields"]["body"][0]
    g["nodes"]["add"]["op_fields"]["body"][0] = body.replace(
        "body=(StridedLoop(",
        "body=(BlockScaleLoad(frag='f', src_buffer='x0', src_index=(), role='a'), StridedLoop(", 1)
    (tmp_path / "k.ir.json").write_text(json.dumps(g))
    (tmp_path / "meta.json").write_text(json.dumps(m))
    r = _cli(str(tmp_path / "k.ir.json"))
    assert r.returncode == 1 and r.stderr.startswith("unsupported construct:")


@pytest.mark.parametrize("name", CONFIGS)
def test_configs_assemble(name, native_lib):
    from emmy_b200 import native
    small = {"vector_add": dict(n=1 << 16), "full_sum": dict(n=1 << 20, ctas=64),
             "row_sum": dict(rows=64, cols=2048), "row_mean": dict(rows=64, cols=2048),
             "rmsnorm": dict(rows=64, cols=1024), "softmax": dict(rows=64, cols=1024),
             "l2norm": dict(rows=64, cols=1024)}
    for kw in ({}, small[name]):
        g, m = synth.config(name, **kw).build()
        c = compile_graph(g, m)
        assert c.kind in ("pointwise", "rows")
        img = native.Image(c.render())
        regs = img.registers()[c.entry]
        assert regs <= 128, regs
        assert "spill" not in img.log or "0 bytes spill stores" in img.log


def test_in_process_api():
    """The names the reference's in-process callers use (tools/harness/regression.py:26-45)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("emmy_compile", REPO / "compile.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    folder = REPO / "tests/golden/problems/r04_row_sum"
    g = mod.Graph.from_dict(json.loads((folder / "kernel.ir.json").read_text()))
    c = mod.Compiler(g, json.loads((folder / "meta.json").read_text()), mod.find_kernel(g))
    c.compile()
    assert c.render() == mod.compile_ir(folder / "kernel.ir.json")


def test_generic_lowering_assembles_all_goldens(native_lib, monkeypatch):
    """Every golden IR (15 problems, 8 bug fixtures) also compiles through the
    statement-by-statement lowering and assembles for sm_100a."""
    from conftest import FIXTURES, PROBLEMS
    from emmy_b200 import native
    monkeypatch.setenv("EMMY_TEMPLATE", "generic")
    for folder in PROBLEMS + FIXTURES:
        g = json.loads((folder / "kernel.ir.json").read_text())
        m = json.loads((folder / "meta.json").read_text())
        c = compile_graph(g, m)
        assert c.kind == "generic"
        native.Image(c.render())


@pytest.mark.parametrize("name", ["attention", "attention_d64"])
@pytest.mark.parametrize("bm", [128, 256])
def test_attention_register_split(name, bm):
    """The attention kernel hands registers between warpgroups with
    setmaxnreg: the assembled function must hold exactly the declared count
    per thread at launch (.maxnreg with setmaxnreg), the shares must add up to
    no more than the launch's registers, and each setmaxnreg must match its
    share (an .inc that asks for more than was freed would wait forever)."""
    import re
    from emmy_b200 import harness, synth
    g, m = synth.config(name, B=1, H=2, S=512, BM=bm).build()
    ck = harness.CompiledKernel(g, m)
    mo = harness._REGSPLIT_RE.search(ck.ptx)
    assert mo, "no regsplit declaration"
    launch, threads = int(mo.group(1)), int(mo.group(2))
    shares = [int(x) for x in mo.group(3).split(",")]
    assert f".maxnreg {launch}" in ck.ptx
    assert ck.image.registers()[ck.entry] == launch
    assert threads == 128 * len(shares) and 128 * sum(shares) <= threads * launch
    incs = {int(x) for x in re.findall(r"setmaxnreg\.inc\.sync\.aligned\.u32 (\d+);", ck.ptx)}
    decs = {int(x) for x in re.findall(r"setmaxnreg\.dec\.sync\.aligned\.u32 (\d+);", ck.ptx)}
    assert incs == {max(shares)} and decs == {min(shares)}
    harness.check_regsplit(ck.ptx, launch)
    with pytest.raises(RuntimeError):
        harness.check_regsplit(ck.ptx, launch - 8)


def _defs_uses(lines):
    """(registers written, registers read) by PTX instruction lines."""
    reg = re.compile(r"%[a-z]+\d+")
    stores = ("st.", "mbarrier.arrive", "mbarrier.init", "tcgen05.st", "tcgen05.mma",
              "tcgen05.commit", "tcgen05.dealloc", "cp.async", "bar", "prefetch", "fence",
              "tcgen05.fence", "tcgen05.wait", "red.", "bra", "ret")
    d, u = set(), set()
    for ln in lines:
        s = ln.strip()
        if not s or s.startswith(("//", "$", ".")):
            continue
        g = re.match(r"^@!?(%p\d+)\s+", s)
        if g:
            u.add(g.group(1))
            s = s[g.end():]
        op, _, rest = s.partition(" ")
        regs = reg.findall(rest)
        if op.startswith("mbarrier.try_wait") or op.startswith("mbarrier.test_wait"):
            d.add(regs[0])
            u.update(regs[1:])
        elif op.startswith(stores):
            u.update(regs)
        elif rest.startswith("{"):
            d.update(reg.findall(rest[:rest.index("}")]))
            u.update(reg.findall(rest[rest.index("}"):]))
        elif regs:
            d.add(regs[0])
            u.update(regs[1:])
    return d, u


@pytest.mark.parametrize("kw", [dict(B=1, H=1, S=128, D=128, BM=128), dict(B=1, H=2, S=512),
                                dict(B=1, H=2, S=512, D=64)])
def test_attention_role_regions_self_contained(kw):
    """After the setmaxnreg split the softmax warps and the other warps run
    under different register limits, in code regions that never merge: every
    register a region reads must be written in that region or in the common
    prologue before the split (a value from the other side would be
    undefined there)."""
    from emmy_b200 import harness, synth
    g, m = synth.attention(**kw).build()
    L = harness.CompiledKernel(g, m).ptx.split("\n")
    first = next(i for i, ln in enumerate(L) if ln.startswith("{"))
    split = next(i for i, ln in enumerate(L) if "bra $L_SOFTMAX_" in ln)
    soft = next(i for i, ln in enumerate(L) if ln.startswith("$L_SOFTMAX_"))
    role_end = next(i for i, ln in enumerate(L) if ln.startswith("$L_TEARDOWN_"))
    common = _defs_uses(L[first:split + 1])[0]
    for lo, hi, extra in ((split + 1, soft, (role_end, len(L))), (soft, role_end, None)):
        lines = L[lo:hi] + (L[extra[0]:extra[1]] if extra else [])
        d, u = _defs_uses(lines)
        assert not sorted(u - d - common), (lo, sorted(u - d - common))


def test_gemm_persistent_selection(native_lib):
    """A 4-stage IR ring (one CTA per SM) selects the persistent pair kernel:
    512 tensor-memory columns, idle clusters beyond the 74 workers, clean
    static checks; 2- and 3-stage rings keep the per-tile pair kernel."""
    from emmy_b200 import native, ptxcheck, racecheck
    for stages, persistent in ((4, True), (3, True), (2, False)):
        g, m = synth.matmul(M=1024, N=1024, K=512, stages=stages).build()
        c = compile_graph(g, m)
        ptx = c.render()
        assert ("persistent CTA pairs" in ptx) == persistent, stages
        assert ptxcheck.check(ptx) == [] and racecheck.check(ptx)[0] == []
        img = native.Image(ptx)
        assert "spill" not in img.log or "0 bytes spill stores" in img.log
        if persistent:
            assert "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32" in ptx
            assert ", 512;" in ptx and "mbarrier.arrive.release.cluster.shared::cluster" in ptx


@pytest.mark.parametrize("kw,pair", [(dict(), True), (dict(M=256, N=256, K=64), True),
                                     (dict(M=128, N=256, K=64), False),
                                     (dict(M=256, N=256, K=256, BN=128, U0=8, U1=32), False)])
def test_gemm_cta_pair_selection_and_assembly(kw, pair, native_lib):
    """bf16 128x256 tiles with an even number of M tiles become CTA pairs
    (cluster of 2, cta_group::2); the rest keep the single-CTA kernel.  Both
    assemble and pass the static checker (which includes its copy-broadcast rule)."""
    from emmy_b200 import native, ptxcheck
    g, m = synth.matmul(**kw).build()
    c = compile_graph(g, m)
    ptx = c.render()
    assert c.kind == "gemm"
    assert ("tcgen05.mma.cta_group::2" in ptx) == pair
    assert (".reqnctapercluster 2, 1, 1" in ptx) == pair
    assert ("// @emmy cluster 2 1 1" in ptx) == pair
    assert ptxcheck.check(ptx) == []
    assert not [f for f in ptxcheck.check(ptx) if f[0] == "no-multicast-load"]
    img = native.Image(ptx)
    assert img.registers()[c.entry] <= 128
    assert "spill" not in img.log or "0 bytes spill stores" in img.log


def test_rows_online_softmax_recognised():
    """The rows template evaluates Emmy's online (max, sum exp) softmax
    accumulation as a max tree then independent exponentials; it recognises
    only that exact structure (synthesised IR and the f02 problem), leaves
    the other row kernels alone, and falls back to the IR's own recurrence
    when the body differs (here: the rescale applied to the wrong operand)."""
    from conftest import PROBLEMS
    g, m = synth.config("softmax", rows=64, cols=1024).build()
    c = compile_graph(g, m)
    assert c.kind == "rows" and c.template.online["max"] == "acc0"
    folder = next(p for p in PROBLEMS if p.name == "f02_row_softmax")
    c = compile_graph(json.loads((folder / "kernel.ir.json").read_text()),
                      json.loads((folder / "meta.json").read_text()))
    assert c.template.online is not None
    for name in ("rmsnorm", "l2norm", "row_sum"):
        gg, mm = synth.config(name, rows=64, cols=1024).build()
        assert compile_graph(gg, mm).template.online is None
    bad = json.loads(json.dumps(g))
    node = next(n for n in bad["nodes"].values() if n["op"] == "KernelOp")
    body = node["op_fields"]["body"][0]
    swapped = body.replace("Assign(name='in0__acc1_sa', op=ElementwiseImpl('multiply'), "
                           "args=('acc1', 'in0__alpha')",
                           "Assign(name='in0__acc1_sa', op=ElementwiseImpl('multiply'), "
                           "args=('acc1', 'in0__beta')", 1)
    assert swapped != body
    node["op_fields"]["body"][0] = swapped
    c = compile_graph(bad, m)
    assert c.kind == "rows" and c.template.online is None


def _interpret(prog, env):
    """Run straight-line integer PTX (the ops ``tile_index`` and ``raster``
    emit, predicates included) over the register values in ``env``."""
    ops = {"div": lambda a, b: a // b, "rem": lambda a, b: a % b,
           "mul": lambda a, b: a * b, "sub": lambda a, b: a - b,
           "add": lambda a, b: a + b, "min": min, "shr": lambda a, b: a >> b,
           "shl": lambda a, b: a << b, "and": lambda a, b: a & b,
           "mad": lambda a, b, c: a * b + c}
    for ins in prog:
        guard = None
        if ins.startswith("@"):
            guard, ins = ins.split(" ", 1)
        op, args = ins.split(" ", 1)
        d, *src = [a.strip() for a in args.split(",")]
        v = [env[x] if x in env else int(x) for x in src]
        if guard and not env[guard.lstrip("@!")] ^ guard.startswith("@!"):
            continue
        base, *mods = op.split(".")
        if base == "setp":
            env[d] = {"ge": v[0] >= v[1], "lt": v[0] < v[1]}[mods[0]]
        elif base == "selp":
            env[d] = v[0] if v[2] else v[1]
        else:
            env[d] = ops[base](*v)
    return env


@pytest.mark.parametrize("MB,NB", [(1, 1), (2, 3), (16, 32), (17, 5), (40, 7), (64, 32), (3, 100),
                                   (8, 32), (4, 20)])
@pytest.mark.parametrize("group", [1, 8, 16])
def test_gemm_raster_is_a_bijection(MB, NB, group):
    """The persistent CTA-pair GEMM's tile order (``gemm_persistent.tile_index``
    then ``raster``, run here by interpreting their emitted integer PTX) walks
    each cluster through the work list of ``cluster_tiles``: full rounds of
    tiles c, c+W, ..., then a leftover tile or a 256 x 128 half of one.  Over
    all clusters every column of every (row band, column block) is computed
    exactly once -- including a last raster group with fewer bands and the
    split tails (8 x 32 = 256 tiles, the matmul shard of one GPU in eight:
    34 leftover tiles become 68 halves of 256 x 128)."""
    from emmy_b200.ptx import Kernel
    from emmy_b200.templates.gemm_persistent import (WORKERS, cluster_tiles, raster, schedule,
                                                     tile_index)
    tiles = MB * NB
    W, NF, R, half = schedule(tiles)
    assert half == ((MB, NB) in {(17, 5), (3, 100), (8, 32), (4, 20)})
    k = Kernel("t", [])
    idx, clus = k.reg("r"), k.reg("r")
    tt, ph_, hoff = tile_index(k, idx, clus, W, NF, half)
    mp, nbk = raster(k, tt, MB, NB, group)
    prog = [ln.strip().rstrip(";") for ln in k.lines]
    cover = {}
    for c in range(W):
        work = cluster_tiles(c, tiles)
        assert len(work) in (NF, NF + 1)
        for i, (t, off, width) in enumerate(work):
            env = _interpret(prog, {idx: i, clus: c})
            assert env[tt] == t
            assert (env[hoff] if half else 0) == off
            if half:
                assert env[ph_] == (width == 128)
            band, blk = env[mp], env[nbk]
            assert 0 <= band < MB and 0 <= blk < NB
            for col in range(off, off + width, 64):
                cover[(band, blk, col)] = cover.get((band, blk, col), 0) + 1
    assert len(cover) == tiles * 4 and set(cover.values()) == {1}


@pytest.mark.parametrize("units,workers", [(512, 148), (4096, 148), (4, 148), (150, 148),
                                           (160, 148), (296, 148), (300, 148), (7, 3)])
@pytest.mark.parametrize("split", [True, False])
def test_attention_units_cover_every_row_once(units, workers, split):
    """The persistent attention schedule (``attention.cta_units``, and its
    emitted form ``unit_rows`` run by interpreting the integer PTX): over all
    worker CTAs every (unit, key) pair is computed exactly once -- a whole
    unit by one CTA, or a split unit's 256 rows by two CTAs over the two
    halves of the keys, only in the last iteration of each.  Key rows are
    the unit's own (batch, head)'s.  512 units on 148 workers is one GPU's
    share of the attention config at 8 GPUs: 3 full rounds and 68 leftover
    units split over 136 CTAs."""
    from emmy_b200.ptx import Kernel
    from emmy_b200.templates.attention import cta_units, unit_rows, unit_schedule
    S, NT = 1024, 2
    QB = S // (128 * NT)
    sched = unit_schedule(units, workers, split)
    W, NF, R, half = sched
    assert half == (split and R > 0 and 2 * R <= W)
    k = Kernel("t", [])
    u, cta = k.reg("r"), k.reg("r")
    q0, k0, ph_ = unit_rows(k, u, cta, sched, QB, S, NT)
    prog = [ln.strip().rstrip(";") for ln in k.lines]
    cover = {}
    for c in range(workers + 2):
        work = cta_units(c, units, workers, split)
        assert (c >= W) == (not work)
        assert all(h is None for _, h in work[:-1])
        for i, (unit, kh) in enumerate(work):
            env = _interpret(prog, {u: i, cta: c})
            bh, qb = divmod(unit, QB)
            assert env[q0] == bh * S + qb * 256
            assert env[k0] == bh * S + (0 if kh is None else kh * S // 2)
            if half:
                assert env[ph_] == (kh is not None)
            for h in ((0, 1) if kh is None else (kh,)):
                cover[(unit, h)] = cover.get((unit, h), 0) + 1
    assert sorted(cover) == [(x, h) for x in range(units) for h in (0, 1)]
    assert set(cover.values()) == {1}


def test_pointwise_batch_follows_the_launch():
    """The pointwise batch (vectors per buffer in flight per thread) grows when
    the IR launches few threads per SM, stays within the register cap, and is
    never larger than a thread's share; loads are coherent (ptxas keeps a
    batch's loads ahead of its stores)."""
    from emmy_b200 import compiler
    from emmy_b200.templates.pointwise import DATA_REGS, batch_size
    assert batch_size(148 * 256, 2, 8) == 8            # one 256-thread CTA per SM
    assert batch_size(148 * 256 * 4, 2, 8) == 4        # four per SM: the minimum
    assert batch_size(148 * 256, 2, 1) == 16           # scalar vectors: the maximum
    for inputs in (1, 2, 3, 5):
        u = batch_size(148 * 32, inputs, 8)
        assert u * inputs * 8 <= max(DATA_REGS, 4 * inputs * 8)
    cases = {(): 4, (("n", 268_435_456),): 8, (("n", 100),): 1}
    for kw, want in cases.items():
        g, m = synth.vector_add(**dict(kw)).build()
        c = compiler.compile_graph(g, m)
        ptx = c.render()
        assert c.template.batch == want, (kw, c.template.batch)
        assert "ld.global.L1::no_allocate." in ptx
        assert "ld.global.nc" not in ptx


def test_tf32_split_with_raw_high_part():
    """3xTF32 with the raw slice as the high part: the tensor core keeps a tf32
    element's top 19 bits, so hi = x & 0xFFFFE000 and the converters write only
    lo = x - hi, which is exact in f32 and below 2^-10 |x|; the persistent
    kernel's converters then hold no tf32 rounding and store one tile, not two."""
    import numpy as np
    from emmy_b200 import compiler
    from emmy_b200.templates import gemm as G
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100_000).astype(np.float32),
                        np.float32([1.0, -1.0, 3.0e-38, 1.0e38, 0.0])])
    hi = (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    lo = (x - hi).astype(np.float32)
    assert np.array_equal((hi.astype(np.float64) + lo.astype(np.float64)).astype(np.float32), x)
    nz = x != 0
    assert np.all(np.abs(lo[nz]) < np.abs(x[nz]) * 2.0 ** -10)
    assert G.TF32_HI_RAW
    g, m = synth.matmul(dtype="f32", BK=32, stages=4, M=512, N=512, K=256).build()
    ptx = compiler.compile_graph(g, m).render()
    assert "cvt.rna.tf32.f32" not in ptx
    assert "and.b32" in ptx and "-8192" in ptx


def test_small_matmuls_with_little_work_a_thread_stay_generic():
    """Emmy's own matmul IRs whose CTAs give each thread fewer than
    ``GemmSmallTemplate.MIN_MACS_PER_THREAD`` multiply-adds (m02: 16, corpus
    mm256: 48, mm64a and mm_rect2: 64, mm128: 1536) lower through the generic
    path, which times faster there; m01 and mm512 (2048) take tcgen05."""
    from conftest import GOLDEN
    want = {("problems", "m01_matmul_512"): "gemm", ("problems", "m02_matmul_rect"): "generic",
            ("corpus", "mm128"): "generic", ("corpus", "mm256"): "generic",
            ("corpus", "mm512"): "gemm", ("corpus", "mm64a"): "generic",
            ("corpus", "mm_rect2"): "generic"}
    for (sub, name), kind_ in want.items():
        f = GOLDEN / sub / name
        c = compile_graph(json.loads((f / "kernel.ir.json").read_text()),
                          json.loads((f / "meta.json").read_text()))
        assert c.kind == kind_, (name, c.kind, c.rejections)


def test_meta_only_gemm_takes_only_meta_parameters(monkeypatch):
    """Emmy's own matmul IRs (m01, m02, corpus mm*) compile to the tcgen05
    kernel whose parameters are exactly meta ``arg_order`` (no tensor-map
    directives or trailing parameters); with EMMY_META_ONLY=1 the benchmark's
    matmul IRs do too, and attention falls back to the generic lowering."""
    import re
    from conftest import GOLDEN
    from emmy_b200 import synth
    folders = [GOLDEN / "problems" / "m01_matmul_512", GOLDEN / "problems" / "m02_matmul_rect"] + \
        [GOLDEN / "corpus" / n for n in ("mm128", "mm256", "mm512", "mm64a", "mm_rect2")]
    cases = [(json.loads((f / "kernel.ir.json").read_text()),
              json.loads((f / "meta.json").read_text())) for f in folders]
    from emmy_b200.templates.gemm_small import GemmSmallTemplate
    monkeypatch.setattr(GemmSmallTemplate, "MIN_MACS_PER_THREAD", 0)   # every IR on tcgen05
    monkeypatch.setenv("EMMY_META_ONLY", "1")
    cases += [synth.config(n).build() for n in ("matmul_bf16", "matmul_f32")]
    for g, m in cases:
        c = compile_graph(g, m)
        ptx = c.render()
        assert type(c.template).__name__ == "GemmSmallTemplate", c.rejections
        assert "@emmy tmap" not in ptx and "tensormap" not in ptx
        params = re.findall(r"\.param \.(\w+) param_(\w+)", ptx)
        assert [n for _, n in params] == m["kernels"][0]["arg_order"]
    g, m = synth.attention(B=1, H=1, S=256, D=64).build()
    assert compile_graph(g, m).kind == "generic"
    for name in ("a01_attention", "a02_attention_128"):
        f = GOLDEN / "problems" / name
        g, m = json.loads((f / "kernel.ir.json").read_text()), json.loads((f / "meta.json").read_text())
        c = compile_graph(g, m)
        assert type(c.template).__name__ == "AttentionSmallTemplate", c.rejections
        params = re.findall(r"\.param \.(\w+) param_(\w+)", c.render())
        assert [n for _, n in params] == m["kernels"][0]["arg_order"]


def test_vocabulary_nodes_lower(native_lib):
    """Pre/Carry, Select and ZeroPrologue (defined by the IR vocabulary,
    lowered by no reference code) go through the statement-by-statement
    lowering, assemble for sm_100a and pass the static checks; a Pre of a
    cell no Carry sets, or a cell indexed at run time, is refused."""
    from emmy_b200 import native, ptxcheck, synth
    from emmy_b200 import ir as I
    for p in (synth.carried_prefix(), synth.carried_prefix(cols=200, every=3),
              synth.select_branches(), synth.zero_prologue()):
        g, m = p.build()
        c = compile_graph(g, m)
        assert c.kind == "generic"
        ptx = c.render()
        native.Image(ptx)
        assert not ptxcheck.check(ptx)
    p = synth.carried_prefix()
    p.body = synth.tile([synth.axis("a0", 64)], [I.Pre("v", "nothing", ()),
                                               synth.write("y", (synth.V("a0"), synth.Lit(0)),
                                                           ("v",))])
    with pytest.raises(NotImplementedError):
        compile_graph(*p.build()).render()


def test_fused_full_sum_variant():
    """``peer_finish`` in the launch descriptor: the split full sum takes the
    four cross-GPU parameters after meta arg_order, declares them in its
    ``// @emmy peer`` line, and passes the static checks; any other kernel
    refuses the request (exit 1) instead of ignoring it."""
    from emmy_b200 import peer, ptxcheck
    from emmy_b200.harness import parse_peer
    g, m = synth.config("full_sum", n=1 << 20, ctas=64).build()
    m["kernels"][0]["peer_finish"] = True
    c = compile_graph(g, m)
    assert c.kind == "rows"
    assert parse_peer(c.ptx) == [n for n, _ in peer.FUSED_PARAMS]
    for n, ty in peer.FUSED_PARAMS:
        assert f".param .{ty} param_{n}" in c.ptx
    assert "st.release.sys.global.u64" in c.ptx and "ld.acquire.sys.global.u64" in c.ptx
    assert ptxcheck.check(c.ptx) == []
    g, m = synth.config("row_sum", rows=64, cols=2048).build()
    m["kernels"][0]["peer_finish"] = True
    with pytest.raises(NotImplementedError):
        compile_graph(g, m)

#!/usr/bin/env python3
"""Benchmark of the reductions configuration.

One step = the three reduction kernels of the configuration, each compiled
by compile.py from an IR in Emmy's schedule form and launched through the C
ABI library (include/emmy_b200.h):

* full-array sum of x_sum, N = 268,435,456 f32 ~ U(0,1) (1 GiB), split form
  (one CTA per ``_ksplit`` chunk, one atomic per CTA, output re-zeroed per
  launch as ``zero_outputs`` says);
* row sum and row mean of x_rows [32768, 8192] f32 ~ N(0,1) (1 GiB).

Metric: achieved HBM throughput (algorithmic bytes: every input read once,
every output written once) over all ranks, in GB/s; ``roofline`` compares the
dominant kernel with the measured copy bandwidth of MEASURED_PEAKS.json.
Multi-GPU (torchrun, one process per GPU): weak scaling -- every rank owns a
full-size shard of each input (its own seed); the full sum finishes with one
NCCL all-reduce of the per-rank partial, inside the step.

Every timed kernel is checked in the same run, after its timing: its module's
``__emmy_status`` word (set when a bounded wait expired) and sampled outputs
against the CPU oracle (``oracle/expr.py``, the checker only) at the
configuration's tolerance; a case that fails reports no number.  After the
headline, N=1 times every other category at its BASELINE size (``categories``,
each with a bounded CPU baseline); N>1 times every configuration as strong
scaling of the BASELINE problem (``shards``: rows, element chunks, CTA slices
of the full sum finished by the all-reduce -- and again by ``peer.PeerSum``,
the same finish over NVLink peer memory without NCCL, and by the sum kernel
itself, whose last CTA runs that exchange (one kernel a rank) -- 256-row bands of
matmul, (batch, head) pairs of attention).  Inputs smaller than twice the L2
are flushed between launches (a 512 MiB write whose lines are then discarded
from L2).

``--impl reference`` times the reference's own CPU evaluation of the same
expressions (numpy, as in the reference's tools/harness/refs.py:41-124) on
the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "emmy-hackathon-2026_b200"))

METRIC = "per-kernel HBM GB/s as % of B200 roofline (reductions: full sum + row sum + row mean)"
WORKLOAD = "reductions: sum(x[268435456] ~ U(0,1)) + x[32768,8192].sum(-1) + x.mean(-1), f32"
FALLBACK_HBM = 6650.0
FALLBACK_BF16 = 1590.0
STEP_BYTES = 3_221_487_624          # full sum + row sum + row mean, per rank


def config_of(world: int) -> dict:
    """The workload description, identical in both arms' JSON lines."""
    return {"workload": WORKLOAD, "step": "one pass of the three reductions",
            "per_rank_bytes_per_step": STEP_BYTES,
            "l2": "each input is 1 GiB > 126 MB L2; no flush needed",
            "parallelism": f"weak scaling over {world} rank(s); full sum finished by "
                           "NCCL all-reduce"}


def peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM, "fallback"


def profile_traffic(config: str):
    """DRAM bytes per launch from the committed ncu summary of that
    configuration's kernel (``profiles/<config>__<entry>.md``, line
    ``traffic_bytes_per_launch: N``); None when no capture exists."""
    for f in sorted((REPO / "profiles").glob(f"{config}__*.md")):
        for ln in f.read_text().splitlines():
            if ln.strip().startswith("traffic_bytes_per_launch:"):
                try:
                    return int(ln.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


class Clocks:
    """nvidia-smi sampled during the timed region (clocks and throttle reasons)."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_problems():
    from emmy_b200 import synth
    return [("full_sum", synth.full_sum()), ("row_sum", synth.row_reduce(mean=False)),
            ("row_mean", synth.row_reduce(mean=True))]


def bytes_of(p) -> int:
    from emmy_b200 import synth
    return synth.algorithmic_bytes(p)


def bf16_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return FALLBACK_BF16, "fallback"


# --------------------------------------------------------------------------
# CPU evaluation (the reference's numpy expressions)
# --------------------------------------------------------------------------

def cpu_reductions(x_sum, x_rows, threads: int = 1) -> float:
    """Seconds for one pass of the three numpy reductions (refs.py's
    ``v["x"].sum()``, ``.sum(-1)``, ``.mean(-1)`` on float32 inputs), split
    over ``threads`` workers by contiguous chunks (numpy releases the GIL)."""
    import numpy as np
    t0 = time.perf_counter()
    if threads <= 1:
        np.sum(x_sum)
        x_rows.sum(-1)
        x_rows.mean(-1)
    else:
        with ThreadPoolExecutor(threads) as ex:
            parts = list(ex.map(np.sum, np.array_split(x_sum, threads)))
            float(np.sum(parts))
            list(ex.map(lambda a: a.sum(-1), np.array_split(x_rows, threads)))
            list(ex.map(lambda a: a.mean(-1), np.array_split(x_rows, threads)))
    return time.perf_counter() - t0


def host_inputs(rank: int):
    import torch
    from emmy_b200.dist import rank_seed
    g = torch.Generator().manual_seed(rank_seed(0, rank))
    x_sum = torch.rand(268_435_456, generator=g, dtype=torch.float32)
    g.manual_seed(rank_seed(1, rank))
    x_rows = torch.randn(32768, 8192, generator=g, dtype=torch.float32)
    return x_sum, x_rows


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    x_sum, x_rows = host_inputs(0)
    xs, xr = x_sum.numpy(), x_rows.numpy()
    threads = len(os.sched_getaffinity(0))
    probs = make_problems()
    total = sum(bytes_of(p) for _, p in probs)
    for _ in range(args.warmup):
        cpu_reductions(xs, xr, threads)
    ts = [cpu_reductions(xs, xr, threads) for _ in range(args.steps)]
    sec = sum(ts) / len(ts)
    v = total / sec / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_of(world),
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads,
                             "kind": "port",
                             "sample": "full workload (3 GiB read), numpy reductions split "
                                       f"over {threads} threads"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_case(name: str) -> dict | None:
    """The category's CPU baseline on a bounded sample of its BASELINE
    workload, timed on this host (median of 3 after one warm pass): numpy
    float32 expressions single-threaded for the pointwise add and the fused row
    ops (the reference's refs.py forms), numpy/OpenBLAS float32 matmul on every
    host core, torch CPU ``scaled_dot_product_attention`` in fp32 on every host
    core.  Returns the metric of the category (GB/s or TFLOP/s)."""
    import numpy as np
    cores = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(0)

    def timed(fn, reps=3):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    if name in ("vector_add", "vector_add_large"):
        n = 1_048_576 if name == "vector_add" else 1 << 25
        a = rng.uniform(-1, 1, n).astype(np.float32)
        b = rng.uniform(-1, 1, n).astype(np.float32)
        sec = timed(lambda: a + b, 20 if n < 1 << 22 else 3)
        return {"value": round(12 * n / sec / 1e9, 2), "unit": "GB/s", "cores": 1, "kind": "port",
                "sample": f"a + b over {n} f32 elements (numpy, one thread)"
                          + ("" if name == "vector_add" else "; 1/8 of the 2^28-element case")}
    if name in ("rmsnorm", "softmax", "l2norm"):
        rows, cols = 4096, 4096
        x = rng.standard_normal((rows, cols)).astype(np.float32)
        w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
        fn = {
            "rmsnorm": lambda: x / np.sqrt((x * x).mean(-1, keepdims=True) + np.float32(1e-6)) * w,
            "softmax": lambda: (lambda z: (lambda e: e / e.sum(-1, keepdims=True))(
                np.exp(z - z.max(-1, keepdims=True))))(x * np.float32(4.0)),
            "l2norm": lambda: x / np.maximum(np.sqrt((x * x).sum(-1, keepdims=True)),
                                             np.float32(1e-12)),
        }[name]
        sec = timed(fn)
        return {"value": round(8 * rows * cols / sec / 1e9, 2), "unit": "GB/s", "cores": 1,
                "kind": "port",
                "sample": f"{rows} of the 65536 rows x {cols} (1/16 of the workload), numpy "
                          "float32, one thread"}
    if name in ("matmul_bf16", "matmul_f32"):
        from threadpoolctl import threadpool_limits
        M, N, K = 2048, 8192, 4096
        a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
        with threadpool_limits(limits=cores, user_api="blas"):
            sec = timed(lambda: a @ b)
        return {"value": round(2 * M * N * K / sec / 1e12, 3), "unit": "TFLOP/s", "cores": cores,
                "kind": "port",
                "sample": f"A[{M}, {K}] @ B[{K}, {N}] (1/8 of the M rows), numpy/OpenBLAS "
                          f"float32 sgemm on {cores} threads"
                          + (" (bf16 inputs held as float32)" if name == "matmul_bf16" else "")}
    if name in ("attention", "attention_d64"):
        import torch
        D = 128 if name == "attention" else 64
        H, S = 4, 4096
        torch.set_num_threads(cores)
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(1, H, S, D, generator=g) for _ in range(3))
        sec = timed(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v))
        return {"value": round(4 * H * S * S * D / sec / 1e12, 3), "unit": "TFLOP/s",
                "cores": cores, "kind": "port",
                "sample": f"{H} of the 256 (batch, head) pairs, S={S}, d={D}: torch CPU "
                          f"scaled_dot_product_attention fp32 on {cores} threads"}
    return None


# --------------------------------------------------------------------------
# same-run checks
# --------------------------------------------------------------------------

def read_status(kern) -> int | None:
    """The module's ``__emmy_status`` word (nonzero once a bounded wait has
    expired in any launch of the module); None for kernels without one."""
    import torch
    from emmy_b200 import native
    try:
        addr, _ = kern.module().global_addr("__emmy_status")
    except native.EmmyError:
        return None
    st = torch.zeros(1, dtype=torch.int32)
    native.check(native.lib().emmy_memcpy_dtoh_async(st.data_ptr(), addr, 4, None))
    torch.cuda.synchronize()
    return int(st[0])


def _host(t, dt: str):
    """A device tensor (slice) as the oracle takes it: bf16 as uint16 bits."""
    import numpy as np
    import torch
    if dt == "bf16":
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return t.contiguous().cpu().numpy()


def check_outputs(p, kern, bufs, stream, seed: int = 0) -> dict:
    """Same-run correctness of a kernel that was just timed, outside the timed
    region: one more launch on the timed buffers (outputs zeroed first, as
    ``zero_outputs`` says), the module's status word, and sampled outputs
    against the CPU oracle at the configuration's tolerance (bit-exact for the
    pointwise add).  Samples: the whole output up to 4 Mi elements, else four
    1 Mi-element windows (pointwise); the whole input (full sum); 64 rows (row
    kernels); 16 rows of C (matmul); 2 (batch, head) pairs (attention)."""
    import numpy as np
    import torch
    from emmy_b200 import native
    sys.path.insert(0, str(REPO))
    from oracle import expr

    L = native.lib()
    for z, nb in bufs.zero_list():
        native.check(L.emmy_memset_async(z, 0, nb, stream))
    kern.launch(bufs.ptrs(), stream)
    torch.cuda.synchronize()
    status = read_status(kern) if kern.kind != "ptx" else None
    m = p.meta()
    spec = m["oracle"]
    fam, out = spec["family"], spec["output"]
    args = bufs.args
    rng = np.random.default_rng(seed)

    def dev(name):
        shape = args[name]["shape"]
        return bufs.t[name].view(*shape) if shape else bufs.t[name]

    def host(name, sel=None):
        t = dev(name)
        return _host(t if sel is None else t[sel], args[name]["dtype"])

    names = list(spec["args"].values())
    pairs = []                                   # (inputs, got) samples
    if fam == "add":
        n = args[out]["shape"][0]
        if n <= 1 << 22:
            sels, what = [slice(0, n)], f"all {n} elements"
        else:
            w = 1 << 20
            starts = sorted(int(s) * w for s in rng.choice(n // w, 4, replace=False))
            sels, what = [slice(s0, s0 + w) for s0 in starts], "4 windows of 2^20 elements"
        for sl in sels:
            pairs.append(({x: host(x, sl) for x in names}, host(out, sl)))
    elif fam == "sum":
        what = "the whole input"
        pairs.append(({x: host(x) for x in names}, host(out)))
    elif fam in ("row_sum", "row_mean", "rmsnorm", "softmax", "l2norm"):
        R = args[out]["shape"][0]
        k = min(64, R)
        rows = np.sort(rng.choice(R, k, replace=False))
        idx = torch.as_tensor(rows, device=bufs.t[out].device)
        what = f"{k} sampled rows"
        ins = {}
        for x in names:
            sh = args[x]["shape"]
            ins[x] = host(x, idx) if len(sh) == 2 and sh[0] == R else host(x)
        pairs.append((ins, host(out, idx)))
    elif fam == "matmul":
        Mr = args[out]["shape"][0]
        k = min(16, Mr)
        rows = np.sort(rng.choice(Mr, k, replace=False))
        idx = torch.as_tensor(rows, device=bufs.t[out].device)
        what = f"{k} sampled rows of C"
        a, b = spec["args"]["a"], spec["args"]["b"]
        pairs.append(({a: host(a, idx), b: host(b)}, host(out, idx)))
    elif fam == "attention":
        B, H = args[out]["shape"][:2]
        flat = rng.choice(B * H, min(2, B * H), replace=False)
        bh = [(int(f) // H, int(f) % H) for f in sorted(flat)]
        what = f"(batch, head) pairs {bh}"
        ins = {x: np.stack([host(x, (b_, h_)) for b_, h_ in bh]) for x in names}
        pairs.append((ins, np.stack([host(out, (b_, h_)) for b_, h_ in bh])))
    else:
        return {"checked": False, "reason": f"no sampler for family {fam}"}
    ok, err, scale = True, 0.0, 0.0
    for ins, got in pairs:
        ref = expr.evaluate_family(spec, ins)[out]
        got = np.asarray(got).reshape(ref.shape)
        rtol, atol = expr.tolerance(m, ref)
        if rtol == 0 and atol == 0:
            good = got.tobytes() == ref.tobytes()
        else:
            good = bool(np.allclose(got, ref, rtol=rtol, atol=atol))
        ok = ok and good
        d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        err = max(err, float(np.max(d)) if d.size else 0.0)
        scale = max(scale, float(np.max(np.abs(ref))) if ref.size else 0.0)
    if status not in (None, 0):
        ok = False
    res = {"checked": True, "ok": ok, "status": status, "max_abs_err": err,
           "err_over_max_ref": err / scale if scale else 0.0, "sample": what,
           "tolerance": "bit-exact" if not m.get("rtol") and not m.get("atol")
           else f"rtol {m.get('rtol')}, atol {m.get('atol') if m.get('atol') is not None else 'rtol*max|ref|'}"}
    return res


# --------------------------------------------------------------------------
# GPU path
# --------------------------------------------------------------------------

def run_ours(args, rank: int, world: int, local: int) -> None:
    import numpy as np
    import torch
    from emmy_b200 import dist as D
    from emmy_b200 import harness, native
    sys.path.insert(0, str(REPO))
    from oracle import expr

    torch.cuda.set_device(local)
    native.check(native.lib().emmy_device_init(local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream

    probs = make_problems()
    kerns = {n: harness.CompiledKernel(*p.build()) for n, p in probs}
    nbytes = {n: bytes_of(p) for n, p in probs}
    step_bytes = sum(nbytes.values())
    assert step_bytes == STEP_BYTES

    x_sum_h, x_rows_h = host_inputs(rank)
    x_sum_h, x_rows_h = x_sum_h.pin_memory(), x_rows_h.pin_memory()
    x_sum = x_sum_h.to(dev)
    x_rows = x_rows_h.to(dev)
    x_sum_np, x_rows_np = x_sum_h.numpy(), x_rows_h.numpy()
    count = torch.tensor([8192.0], device=dev)
    out_sum = torch.zeros(1, device=dev)
    out_rs = torch.zeros(32768, device=dev)
    out_rm = torch.zeros(32768, device=dev)
    ptrs = {
        "full_sum": {"x": x_sum.data_ptr(), "sum_1": out_sum.data_ptr()},
        "row_sum": {"x": x_rows.data_ptr(), "sum_1": out_rs.data_ptr()},
        "row_mean": {"mean_count": count.data_ptr(), "x": x_rows.data_ptr(),
                     "mean": out_rm.data_ptr()},
    }
    params = {n: kerns[n].params(ptrs[n]) for n in kerns}
    L = native.lib()
    order = ["full_sum", "row_sum", "row_mean"]

    def launch(n):
        k = kerns[n]
        native.check(L.emmy_launch(k.kernel().h, native.u32x3(k.grid), native.u32x3(k.block),
                                   k.smem, k._cluster_arg(), params[n][0], sh))

    def step(evs=None):
        native.check(L.emmy_memset_async(out_sum.data_ptr(), 0, 4, sh))
        for i, n in enumerate(order):
            if evs is not None:
                evs[i].record(stream)
            launch(n)
        if evs is not None:
            evs[3].record(stream)
        D.global_sum(out_sum)

    # the oracle's float64 sum (``expr.full_sum`` before its float32 cast) of
    # this rank's input, and of all ranks' inputs: each rank's float64
    # partial, all-reduced in float64
    own64 = float(np.sum(x_sum_np, dtype=np.float64))
    part64 = torch.tensor([own64], dtype=torch.float64, device=dev)
    D.global_sum(part64)
    ref_total = float(part64.item())
    sample_rows = np.sort(np.random.default_rng(5 + rank).choice(32768, 64, replace=False))
    ref_rs = expr.row_sum(x_rows_np[sample_rows])
    ref_rm = expr.row_mean(x_rows_np[sample_rows])

    def check_headline(tag: str) -> dict:
        """The step's three outputs against the oracle (the all-reduced full
        sum against the sum of every rank's input)."""
        got_sum = float(out_sum.item())
        rs = out_rs.cpu().numpy()[sample_rows]
        rm = out_rm.cpu().numpy()[sample_rows]
        rel_sum = abs(got_sum - ref_total) / abs(ref_total)
        ok_rs = np.allclose(rs, ref_rs, rtol=1e-4, atol=1e-4 * float(np.abs(ref_rs).max()))
        ok_rm = np.allclose(rm, ref_rm, rtol=1e-4, atol=1e-4 * float(np.abs(ref_rm).max()))
        res = {"checked": True, "ok": bool(rel_sum <= 1e-4 and ok_rs and ok_rm),
               "full_sum_rel_err": rel_sum,
               "row_sum_max_abs_err": float(np.abs(rs - ref_rs).max()),
               "row_mean_max_abs_err": float(np.abs(rm - ref_rm).max()),
               "sample": f"full sum of all {world} rank(s)' inputs; 64 sampled rows of the "
                         "row kernels", "tolerance": "rtol 1e-4"}
        assert res["ok"], (tag, res)
        return res

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    D.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        start.record(stream)
        for s in range(args.steps):
            step(evs[s])
        end.record(stream)
        torch.cuda.synchronize()
    D.barrier()
    ms = start.elapsed_time(end)
    per = {n: [evs[s][i].elapsed_time(evs[s][i + 1]) for s in range(args.steps)]
           for i, n in enumerate(order)}
    ms_max = D.max_over_ranks(ms, device=dev)
    value = step_bytes * world * args.steps / (ms_max / 1e3) / 1e9
    # the last timed step's outputs (the all-reduced sum included)
    headline_check = check_headline("headline")

    # e2e through the C ABI with host buffers: copies in, launch, result out
    host_out = {"full_sum": np.zeros(1, np.float32), "row_sum": np.zeros(32768, np.float32),
                "row_mean": np.zeros(32768, np.float32)}
    host = {
        "full_sum": {"x": x_sum_np, "sum_1": host_out["full_sum"]},
        "row_sum": {"x": x_rows_np, "sum_1": host_out["row_sum"]},
        "row_mean": {"mean_count": np.array([8192.0], np.float32), "x": x_rows_np,
                     "mean": host_out["row_mean"]},
    }
    devt = {
        "full_sum": {"x": x_sum, "sum_1": out_sum},
        "row_sum": {"x": x_rows, "sum_1": out_rs},
        "row_mean": {"mean_count": count, "x": x_rows, "mean": out_rm},
    }
    e2e_steps = args.steps
    # a step's inputs cross PCIe once: x_rows feeds both row kernels, so the
    # second call finds it resident (copied earlier in the same step)
    from emmy_b200.data import nbytes as nb
    resident, h2d, d2h = {}, 0, 0
    seen = set()
    for n in order:
        resident[n] = set()
        for a in kerns[n].info["args"]:
            if a.get("output"):
                d2h += nb(a)
                continue
            key = (host[n][a["name"]].ctypes.data, devt[n][a["name"]].data_ptr())
            if key in seen:
                resident[n].add(a["name"])
            else:
                seen.add(key)
                h2d += nb(a)
    for n in order:  # warm
        harness.run_host(kerns[n], host[n], devt[n], sh, resident[n])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    D.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        for n in order:
            harness.run_host(kerns[n], host[n], devt[n], sh, resident[n])
        D.global_sum(out_sum)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = D.max_over_ranks(e0.elapsed_time(e1), device=dev)
    e2e_val = step_bytes * world * e2e_steps / (e2e_ms / 1e3) / 1e9
    # the host outputs of the end-to-end path against the oracle (row kernels
    # on the input the step copied once; the per-rank sum before its
    # all-reduce, which runs on the device copy)
    e2e_ok = (np.allclose(host_out["row_sum"][sample_rows], ref_rs, rtol=1e-4,
                          atol=1e-4 * float(np.abs(ref_rs).max()))
              and np.allclose(host_out["row_mean"][sample_rows], ref_rm, rtol=1e-4,
                              atol=1e-4 * float(np.abs(ref_rm).max()))
              and abs(float(host_out["full_sum"][0]) - own64) <= 1e-4 * abs(own64))
    assert e2e_ok, "end-to-end outputs differ from the oracle"

    # reference compiler's PTX for the same IRs, JIT-run on this GPU, each
    # checked against the oracle after its timing
    ref_ptx, ref_ok = {}, {}
    for n in order:
        f = REPO / "oracle" / "_ref" / f"{n}.ptx"
        if not f.exists():
            continue
        import ctypes
        k = kerns[n]
        ref = harness.CompiledKernel.from_ptx(f.read_text(), dict(k.info, entry="ref_" + k.entry))
        kh = ref.kernel()
        arr, keep = ref.params(ptrs[n])
        zero = [(out_sum.data_ptr(), 4)] if n == "full_sum" else []
        it = 10
        outbuf = (ctypes.c_float * it)()
        zd = (ctypes.c_uint64 * 1)(*([z[0] for z in zero] or [0]))
        zb = (ctypes.c_size_t * 1)(*([z[1] for z in zero] or [0]))
        native.check(L.emmy_time_launches(kh.h, native.u32x3(k.grid), native.u32x3(k.block),
                                          k.smem, None, arr, sh, 2, it, 0, 0, zd, zb,
                                          len(zero), outbuf))
        torch.cuda.synchronize()
        if n == "full_sum":
            good = abs(float(out_sum.item()) - own64) <= 1e-4 * abs(own64)
        else:
            got = (out_rs if n == "row_sum" else out_rm).cpu().numpy()[sample_rows]
            want = ref_rs if n == "row_sum" else ref_rm
            good = bool(np.allclose(got, want, rtol=1e-4, atol=1e-4 * float(np.abs(want).max())))
        ref_ok[n] = good
        if good:
            ref_ptx[n] = statistics.median(list(outbuf))
        ref._module.unload()
        del keep
    ours_med = {n: statistics.median(per[n]) for n in order}

    hbm, src = peaks()
    dom = max(order, key=lambda n: sum(per[n]))
    avg = sum(per[dom]) / len(per[dom])
    achieved = nbytes[dom] / (avg / 1e3) / 1e9
    traffic = profile_traffic(dom)
    cats = {}
    for n in order:
        a = sum(per[n]) / len(per[n])
        gbs = nbytes[n] / (a / 1e3) / 1e9
        cats[n] = {"ms": round(a, 4), "GB/s": round(gbs, 1), "frac": round(gbs / hbm, 3)}
        if n in ref_ptx:
            cats[n]["reference_ptx_ms"] = round(ref_ptx[n], 4)
            cats[n]["speedup_vs_reference_ptx"] = round(ref_ptx[n] / ours_med[n], 2)
        if n in ref_ok:
            cats[n]["reference_ptx_checked"] = ref_ok[n]
    cpu = None
    if rank == 0 and world == 1:
        cpu_reductions(x_sum_np, x_rows_np, 1)
        ts = [cpu_reductions(x_sum_np, x_rows_np, 1) for _ in range(3)]
        sec = statistics.median(ts)
        cpu = {"value": round(step_bytes / sec / 1e9, 3), "unit": "GB/s", "cores": 1,
               "kind": "port",
               "sample": "full workload once per run (median of 3), numpy float32 reductions "
                         "as the reference's refs.py, single thread"}
    categories = cat_clocks = None
    if world == 1 and not args.no_categories:
        # every other category's kernel at its BASELINE size (own buffers;
        # the reductions inputs are released first)
        del x_sum, x_rows, devt, host, ptrs, params
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        categories = {}
        with Clocks(local) as cclk:
            for nm in CATEGORY_CASES:
                try:
                    # 10 launches as a burst, comparable with the burst peaks
                    # (longer runs of the contractions settle at the
                    # power-capped clock); the microsecond-scale vector add
                    # takes 50 for a stable median
                    r = measure_case(nm, {}, 50 if nm == "vector_add" else 10, 3,
                                     extras=nm == "vector_add")
                except Exception as e:  # report, keep the headline line
                    categories[nm] = {"error": f"{type(e).__name__}: {e}"[:300]}
                    continue
                categories[nm] = {kk: r[kk] for kk in (
                    "template", "ms_median", "GB/s", "TFLOP/s", "frac", "peak_basis",
                    "reference_ptx_ms", "speedup_vs_reference_ptx", "reference_ptx_check",
                    "check", "back_to_back", "rotated", "wide_launch") if kk in r}
        cat_clocks = cclk.summary()
        if rank == 0:
            for nm in CATEGORY_CASES:
                try:
                    categories[nm]["cpu_baseline"] = cpu_case(nm)
                except Exception as e:
                    categories[nm]["cpu_baseline"] = {"error": f"{type(e).__name__}: {e}"[:200]}
    shards = None
    if world > 1 and not args.no_categories:
        del x_sum, x_rows, devt, host, ptrs, params
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        shards = run_shards(rank, world, dev)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (torch.Generator seeds 1000*rank+{0,1}; BASELINE distributions)",
            "config": config_of(world),
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                         "peak": hbm, "peak_source": src, "unit": "GB/s",
                         "frac": round(achieved / hbm, 3), "traffic": traffic,
                         "algorithmic_bytes": nbytes[dom]},
            "check": headline_check,
            "kernels": cats,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps, "checked": True,
                    "path": "emmy_run_host (C ABI) from pinned host memory"},
            "gpu_launches": 3 * args.steps,
            "clocks": clk.summary(),
            "categories": categories,
            "categories_clocks": cat_clocks,
            "shards": shards,
        }
        print(json.dumps(line), flush=True)


def run_shards(rank: int, world: int, dev) -> dict:
    """Every configuration at N > 1 as strong scaling of its BASELINE problem:
    each rank times its shard (10 launches, median), the job's time is the
    max over ranks, and each rank checks its shard's outputs against the
    oracle; a shard that fails on any rank reports no number."""
    import torch
    from emmy_b200 import dist as D
    from emmy_b200 import synth
    hbm, _ = peaks()
    bf, _ = bf16_peak()
    shards = {}
    for nm in D.SHARDED:
        kw = D.shard_kwargs(nm, rank, world)
        try:
            if nm == "full_sum":
                r = measure_full_sum_strong(kw, 20, 3, dev, rank)
            else:
                r = measure_case(nm, kw, 10, 3, seed=rank)
            ms_r, err = r["ms_median"], None
            ok_r = bool(r["check"]["ok"])
            e_r = float(r["check"]["err_over_max_ref"])
        except Exception as e:  # every rank still joins the reductions below
            r, ms_r, err, ok_r, e_r = None, float("inf"), f"{type(e).__name__}: {e}"[:300], \
                False, float("inf")
        ms_all = D.max_over_ranks(ms_r, device=dev)
        ok_all = D.max_over_ranks(0.0 if ok_r else 1.0, device=dev) == 0.0
        err_all = D.max_over_ranks(e_r, device=dev)
        full = synth.config(nm)
        flops = synth.algorithmic_flops(full)
        d = {"partition": D.SHARDED[nm][0], "rank0_shard": D.shard_kwargs(nm, 0, world),
             "ms_max_over_ranks": round(ms_all, 5) if ok_all else None, "scaling": "strong",
             "check": {"checked": True, "ok_all_ranks": ok_all, "err_over_max_ref_max": err_all,
                       "sample": r["check"]["sample"] if r else None}}
        if ok_all and ms_all < 1e30:
            if flops:
                tf = flops / (ms_all / 1e3) / 1e12
                peak = bf / 6 if nm == "matmul_f32" else bf
                d.update({"TFLOP/s": round(tf, 1), "frac_of_n_peaks": round(tf / (world * peak), 3)})
            else:
                gbs = synth.algorithmic_bytes(full) / (ms_all / 1e3) / 1e9
                d.update({"GB/s": round(gbs, 1), "frac_of_n_peaks": round(gbs / (world * hbm), 3)})
        if err:
            d["error"] = err
        if nm == "full_sum":
            d["collective"] = ("NCCL all-reduce of the per-rank partial, inside each timed step "
                               "(output reset, sum kernel and all-reduce replayed as one CUDA graph)")
            if world > 1:
                d["nvlink_finish"] = peer_finish_shard(kw, world, rank, dev, hbm)
                d["fused_finish"] = peer_finish_shard(kw, world, rank, dev, hbm, fused=True)
        shards[nm] = d
    return shards


def peer_finish_shard(kw: dict, world: int, rank: int, dev, hbm: float,
                      fused: bool = False) -> dict:
    """The strong-scaled full sum with its cross-GPU step done by
    ``peer.PeerSum`` (partials written into every peer's memory over NVLink,
    no collective library), timed and checked like the NCCL form; ``fused``:
    the exchange runs inside the sum kernel (its last CTA), one kernel a
    rank."""
    from emmy_b200 import dist as D
    from emmy_b200 import synth
    try:
        r = measure_full_sum_strong(kw, 20, 3, dev, rank,
                                    exchange="fused" if fused else "nvlink")
        ms_r, ok_r, err = r["ms_median"], bool(r["check"]["ok"]), None
    except Exception as e:  # every rank still joins the reductions below
        r, ms_r, ok_r, err = None, float("inf"), False, f"{type(e).__name__}: {e}"[:300]
    ms_all = D.max_over_ranks(ms_r, device=dev)
    ok_all = D.max_over_ranks(0.0 if ok_r else 1.0, device=dev) == 0.0
    d = {"exchange": ("the sum kernel's last CTA stores the rank's partial into every rank's "
                      "slot over NVLink (CUDA IPC mappings), polls its own slots and sums them "
                      "in rank order: sum and cross-GPU finish in one kernel a rank" if fused else
                      "peer.PeerSum: each rank's partial stored into every rank's slot over "
                      "NVLink (CUDA IPC mappings), one polling kernel per rank, summed in rank "
                      "order; replayed with the sum kernel as one CUDA graph"),
         "ms_max_over_ranks": round(ms_all, 5) if ok_all else None,
         "check": {"checked": True, "ok_all_ranks": ok_all,
                   "status": r["check"]["status"] if r else None}}
    if ok_all and ms_all < 1e30:
        gbs = synth.algorithmic_bytes(synth.config("full_sum")) / (ms_all / 1e3) / 1e9
        d.update({"GB/s": round(gbs, 1), "frac_of_n_peaks": round(gbs / (world * hbm), 3)})
    if err:
        d["error"] = err
    return d


def measure_full_sum_strong(kw: dict, steps: int, warmup: int, dev, rank: int,
                            exchange: str = "nccl") -> dict:
    """The strong-scaled full sum: each rank sums its CTA slices of the global
    input, then the ranks' partials are summed across GPUs -- by one NCCL
    all-reduce (``exchange="nccl"``) or by ``peer.PeerSum``, one kernel per
    rank that writes its partial into every peer's memory over NVLink and
    sums what arrives (``"nvlink"``); both are inside each timed step.  The step (output reset, sum kernel, all-reduce) is captured
    once as a CUDA graph and ``steps`` replays run back to back between one
    pair of CUDA events on the launching stream (after a barrier), so the
    time per step is the device's: no host launch gap between the kernel and
    the collective.  Checked against the float64 sum of all ranks' slices."""
    import numpy as np
    import torch
    from emmy_b200 import dist as D
    from emmy_b200 import harness, native, synth
    p = synth.config("full_sum", **kw)
    g, m = p.build()
    if exchange == "fused":
        m["kernels"][0]["peer_finish"] = True
    kern = harness.CompiledKernel(g, m)
    bufs = harness.Buffers.random(kern, seed=rank)
    stream = torch.cuda.current_stream()
    out = bufs.t["sum_1"]
    L = native.lib()
    k = kern.kernel()
    ps = None
    if exchange in ("nvlink", "fused"):
        from emmy_b200 import peer
        world = D.from_env().world
        try:
            ps = peer.PeerSum(rank, world)
            built = True
        except Exception:
            built = False
        # every rank maps its peers before any rank launches a kernel that
        # waits for the others
        if D.max_over_ranks(0.0 if built else 1.0, device=dev) != 0.0:
            if ps is not None:
                ps.close(barrier=D.barrier)
            else:
                D.barrier()
            raise RuntimeError("peer memory could not be mapped on every rank")
    ptrs = bufs.ptrs()
    if exchange == "fused":
        ptrs.update(ps.fused_values())
    arr, keep = kern.params(ptrs)

    def step():
        sh = torch.cuda.current_stream().cuda_stream
        native.check(L.emmy_memset_async(out.data_ptr(), 0, 4, sh))
        native.check(L.emmy_launch(k.h, native.u32x3(kern.grid), native.u32x3(kern.block),
                                   kern.smem, kern._cluster_arg(), arr, sh))
        if exchange == "nvlink":
            ps.launch(out.data_ptr(), sh)
        elif exchange == "nccl":
            D.global_sum(out)

    for _ in range(warmup):
        step()
    D.barrier()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(warmup):
        graph.replay()
    D.barrier()
    torch.cuda.synchronize()
    # the steps back to back between one event pair (a host synchronisation
    # after every step would put the ranks' host skew into each all-reduce)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = [e0.elapsed_time(e1) / steps]
    # a graph holding NCCL calls is released before the process group is
    del graph
    torch.cuda.synchronize()
    status = None
    if exchange == "fused":
        status = read_status(kern)
    if ps is not None:
        if exchange == "nvlink":
            status = ps.status()
        D.barrier()                  # every rank's kernels are done before unmapping
        ps.close(barrier=D.barrier)
    got = float(out.item())
    part = torch.tensor([float(np.sum(bufs.t["x"].cpu().numpy(), dtype=np.float64))],
                        dtype=torch.float64, device=dev)
    D.global_sum(part)
    want = float(part.item())
    rel = abs(got - want) / abs(want)
    del keep
    return {"ms_median": float(np.median(ms)),
            "check": {"checked": True, "ok": rel <= 1e-4 and not status, "status": status,
                      "rel_err": rel, "err_over_max_ref": rel,
                      "sample": f"the sum finished by {exchange} against the float64 sum of "
                                "every rank's slices"}}


def back_to_back(kern, ptrs: dict, n: int = 100, reps: int = 5) -> float:
    """Per-launch time of ``n`` launches captured back to back in one CUDA
    graph (no flush, no events between them): the device-side rate of a
    launch-latency-bound kernel."""
    import torch
    from emmy_b200 import native
    L = native.lib()
    k = kern.kernel()
    arr, keep = kern.params(ptrs)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        native.check(L.emmy_launch(k.h, native.u32x3(kern.grid), native.u32x3(kern.block),
                                   kern.smem, kern._cluster_arg(), arr, s.cuda_stream))
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=s):
        for _ in range(n):
            native.check(L.emmy_launch(k.h, native.u32x3(kern.grid), native.u32x3(kern.block),
                                       kern.smem, kern._cluster_arg(), arr, s.cuda_stream))
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for _ in range(reps):
        g.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    del g, keep
    return e0.elapsed_time(e1) / (n * reps)


def rotated(p, kern, sets: int = 32, reps: int = 20, seed: int = 0) -> dict:
    """Per-launch time of a small kernel reading cold inputs without an L2
    flush between launches: ``sets`` buffer sets (together more than twice
    the 126 MB L2) used in turn by ``sets`` launches captured back to back in
    one CUDA graph, so every launch reads inputs that ``sets - 1`` other
    launches' traffic has pushed out of L2.  CUDA events around each replay;
    the median over ``reps`` replays, divided by ``sets``.  Then every output
    is filled with 0xFF bytes, the graph replayed once more, and each set's
    output -- what the graph itself wrote -- compared with the oracle (the
    add: bit-exact)."""
    import numpy as np
    import torch
    from emmy_b200 import harness, native
    sys.path.insert(0, str(REPO))
    from oracle import expr

    L = native.lib()
    k = kern.kernel()
    bufs = [harness.Buffers.random(kern, seed=seed + 1 + i) for i in range(sets)]
    params = [kern.params(b.ptrs()) for b in bufs]
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())

    def launch_all():
        for arr, _ in params:
            native.check(L.emmy_launch(k.h, native.u32x3(kern.grid), native.u32x3(kern.block),
                                       kern.smem, kern._cluster_arg(), arr, s.cuda_stream))
    with torch.cuda.stream(s):
        launch_all()                       # loads the module's launch state off the capture
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=s):
        launch_all()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    ms = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        g.replay()
        e1.record(cur)
        e1.synchronize()
        ms.append(e0.elapsed_time(e1) / sets)
    # the graph's own outputs, against the oracle
    m = p.meta()
    spec = m["oracle"]
    out = spec["output"]
    names = list(spec["args"].values())
    for b in bufs:
        b.t[out].view(torch.uint8).fill_(0xFF)
    g.replay()
    torch.cuda.synchronize()
    status = read_status(kern)
    ok = status in (None, 0)
    for b in bufs:
        ins = {x: _host(b.t[x], b.args[x]["dtype"]) for x in names}
        ref = expr.evaluate_family(spec, ins)[out]
        got = _host(b.t[out], b.args[out]["dtype"]).reshape(ref.shape)
        rtol, atol = expr.tolerance(m, ref)
        if rtol == 0 and atol == 0:
            ok = ok and got.tobytes() == ref.tobytes()
        else:
            ok = ok and bool(np.allclose(got, ref, rtol=rtol, atol=atol))
    set_bytes = sum(t.numel() * t.element_size() for t in bufs[0].t.values())
    del g, params, bufs
    torch.cuda.synchronize()
    return {"us_per_launch": round(float(np.median(ms)) * 1e3, 3),
            "sets": sets, "set_bytes": set_bytes,
            "check": {"checked": True, "ok": bool(ok), "status": status,
                      "sample": f"every output of the {sets} sets, written by the graph"}}


def measure_case(name: str, kw: dict, steps: int, warmup: int, seed: int = 0,
                 extras: bool = False) -> dict:
    """Time one synthesised configuration: ``steps`` launches through the C ABI,
    each bracketed by CUDA events on the launching stream; L2 flushed between
    launches when the inputs would fit in it (512 MiB written, then that
    buffer's lines discarded from L2, so the timed launch neither finds its
    inputs in L2 nor pays the flush's write-back).  Then, outside the timing, the
    outputs are checked (``check_outputs``); a failed check drops the numbers.
    Includes the reference compiler's PTX for the same IR (``oracle/_ref``)
    when it exists, checked the same way.  ``extras`` (the vector add): the
    same kernel back to back in a CUDA graph, and a wider launch of the same
    IR (one 32-byte vector per thread)."""
    import numpy as np
    import torch

    from emmy_b200 import harness, synth

    p = synth.config(name, **kw)
    g, m = p.build()
    kern = harness.CompiledKernel(g, m)
    bufs = harness.Buffers.random(kern, seed=seed)
    stream = torch.cuda.current_stream().cuda_stream
    in_bytes = sum(t.numel() * t.element_size() for n, t in bufs.t.items()
                   if not bufs.args[n].get("output"))
    flush = fb = None
    if in_bytes < 2 * 126 * 2 ** 20:
        fb = torch.empty(512 * 2 ** 20, dtype=torch.uint8, device="cuda")
        flush = (fb.data_ptr(), fb.numel())
    ms = kern.time(bufs.ptrs(), warmup=warmup, iters=steps, stream=stream,
                   flush=flush, zero=bufs.zero_list())
    chk = check_outputs(p, kern, bufs, stream, seed=seed)
    med = float(np.median(ms))
    hbm, src = peaks()
    nb = synth.algorithmic_bytes(p)
    flops = synth.algorithmic_flops(p)
    line = {"case": name, "size": kw, "template": kern.kind, "entry": kern.entry,
            "ms_median": round(med, 5), "ms_min": round(float(np.min(ms)), 5),
            "launches": steps,
            "l2_flush": ("512 MiB written, then discarded from L2" if flush is not None
                         else "inputs larger than twice the L2"),
            "regs": kern.image.registers().get(kern.entry), "check": chk}
    if flops:
        tf = flops / (med / 1e3) / 1e12
        peak, psrc = bf16_peak()
        basis = f"{psrc} bf16 peak"
        if kern.kind == "gemm" and getattr(kern.compiler.template, "mode", "") == "tf32x3":
            # fp32 through 3xTF32: tf32 runs at half the bf16 rate and every
            # product costs three tf32 MMAs
            peak, basis = peak / 2 / 3, f"3xTF32 effective = {psrc} bf16 peak / 2 / 3"
            # the tensor work itself: three tf32 products per multiply-add
            line["raw_tf32"] = {"TFLOP/s": round(3 * tf, 1), "peak": round(3 * peak, 1),
                                "frac": round(tf / peak, 3),
                                "basis": f"{psrc} bf16 peak / 2 (the tf32 rate)"}
        line.update({"TFLOP/s": round(tf, 1), "peak": round(peak, 1), "peak_basis": basis,
                     "frac": round(tf / peak, 3), "flops": flops})
    else:
        gbs = nb / (med / 1e3) / 1e9
        line.update({"GB/s": round(gbs, 1), "peak": hbm, "peak_source": src,
                     "frac": round(gbs / hbm, 3), "algorithmic_bytes": nb})
    if extras and kern.kind == "pointwise":
        t = back_to_back(kern, bufs.ptrs())
        line["back_to_back"] = {"us_per_launch": round(t * 1e3, 3),
                                "GB/s": round(nb / (t / 1e3) / 1e9, 1),
                                "note": "100 launches in one CUDA graph, no L2 flush: the "
                                        "8 MiB of inputs stay in L2 between launches"}
        rot = rotated(p, kern, seed=seed)
        if rot["check"]["ok"]:
            tr = rot["us_per_launch"] / 1e6
            rot.update({"GB/s": round(nb / tr / 1e9, 1), "frac": round(nb / tr / 1e9 / hbm, 3)})
        rot["note"] = ("launches back to back in one CUDA graph over buffer sets used in turn "
                       "(more than twice the L2 between two uses of a set): cold inputs, "
                       "no flush between launches")
        line["rotated"] = rot
        n = p.meta()["kernels"][0]["args"][0]["shape"][0]
        wide = synth.config(name, **{**kw, "threads": max(256, n // 8)})
        wk = harness.CompiledKernel(*wide.build())
        wb = harness.Buffers.random(wk, seed=seed)
        wms = wk.time(wb.ptrs(), warmup=warmup, iters=steps, stream=stream, flush=flush,
                      zero=wb.zero_list())
        wchk = check_outputs(wide, wk, wb, stream, seed=seed)
        wmed = float(np.median(wms))
        line["wide_launch"] = {"grid": list(wk.grid), "block": list(wk.block),
                               "ms_median": round(wmed, 5),
                               "GB/s": round(nb / (wmed / 1e3) / 1e9, 1) if wchk["ok"] else None,
                               "check": wchk}
        del wb
    f = REPO / "oracle" / "_ref" / f"{name}.ptx"
    if f.exists() and not kw:
        # the reference compiler's PTX for the same IR, launched under the same
        # meta entry from its own text (its parameters are the meta arguments
        # alone: no tensor maps, no cluster)
        ref = harness.CompiledKernel.from_ptx(f.read_text(),
                                              dict(kern.info, entry="ref_" + kern.entry))
        rms = ref.time(bufs.ptrs(), warmup=2, iters=min(steps, 10), stream=stream,
                       flush=flush, zero=bufs.zero_list())
        rchk = check_outputs(p, ref, bufs, stream, seed=seed)
        line["reference_ptx_check"] = {"ok": rchk["ok"], "max_abs_err": rchk["max_abs_err"]}
        if rchk["ok"]:
            line["reference_ptx_ms"] = round(float(np.median(rms)), 5)
            line["speedup_vs_reference_ptx"] = round(float(np.median(rms)) / med, 2)
        ref._module.unload()
    if not chk["ok"]:
        for key in ("TFLOP/s", "GB/s", "frac", "speedup_vs_reference_ptx"):
            line.pop(key, None)
        line["error"] = "output check failed: numbers withheld"
    del bufs, fb
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return line


CATEGORY_CASES = ["vector_add", "vector_add_large", "rmsnorm", "softmax", "l2norm", "matmul_bf16",
                  "matmul_f32", "attention", "attention_d64"]


# the reference's own published kernel times for its open problems (H200,
# docs/ATTRIBUTION_PLAYBOOK.md:271-274 of the reference), for comparison only
PUBLISHED_H200_US = {"m01_matmul_512": 15.04, "a01_attention": 47.78, "r03_mean": 6.848,
                     "r02_big_sum": 15.73}


def run_problems(args) -> None:
    """``--problems``: the reference's 15 open problems (their own IRs, meta
    and expected.npz) through this build's compiler and through the
    reference compiler's PTX for the same IRs (``oracle/_ref/problems``),
    both on this GPU: every kernel checked against expected.npz within the
    problem's rtol/atol, then timed (``--steps`` launches back to back, CUDA
    events around each, median).  One JSON line."""
    import torch
    from emmy_b200 import native, problem
    torch.cuda.set_device(0)
    native.check(native.lib().emmy_device_init(0))
    rows = {}
    root = REPO / "tests" / "golden" / "problems"
    for folder in sorted(p for p in root.iterdir() if (p / "meta.json").exists()):
        pid = folder.name
        row = {}
        for arm in ("ours", "ours_generic", "reference_ptx"):
            if arm == "ours":
                rep = problem.run_problem(folder, out=lambda s_: None, time_launches=True,
                                          iters=args.steps)
            elif arm == "ours_generic":
                # the same IRs forced through the statement-by-statement
                # lowering (only where a template was selected)
                if all(k_["kind"] == "generic" for k_ in row["ours"]["kernels"]):
                    continue
                os.environ["EMMY_TEMPLATE"] = "generic"
                try:
                    rep = problem.run_problem(folder, out=lambda s_: None, time_launches=True,
                                              iters=args.steps)
                finally:
                    del os.environ["EMMY_TEMPLATE"]
            else:
                rdir = REPO / "oracle" / "_ref" / "problems" / pid
                if not rdir.exists():
                    continue
                rep = problem.run_problem(
                    folder, ptx_for=lambda k_, ir_: (rdir / f"{k_['entry']}.ptx").read_text(),
                    out=lambda s_: None, time_launches=True, iters=args.steps)
            ks = rep["kernels"]
            row[arm] = {"ok": bool(rep["ok"]),
                        "kernels": [{"entry": k_["entry"], "kind": k_["kind"],
                                     "us": round(k_["us"], 3) if k_["us"] else None} for k_ in ks],
                        "us": round(sum(k_["us"] or 0 for k_ in ks), 3) if rep["ok"] else None}
        if row.get("ours", {}).get("us") and row.get("reference_ptx", {}).get("us"):
            row["speedup_vs_reference_ptx"] = round(row["reference_ptx"]["us"] / row["ours"]["us"], 2)
        if pid in PUBLISHED_H200_US:
            row["reference_published_h200_us"] = PUBLISHED_H200_US[pid]
        rows[pid] = row
    print(json.dumps({"problems": rows, "launches_timed": args.steps,
                      "protocol": "inputs resident; one checked launch, then back-to-back "
                                  "launches with CUDA events around each, no L2 flush "
                                  "(the inputs are at most 1 MiB)"}), flush=True)


def run_case(args) -> None:
    """``--case`` (sizes from ``--size k=v,..``): one JSON line for one
    configuration (per-category numbers; small ncu captures)."""
    import torch

    from emmy_b200 import native

    torch.cuda.set_device(0)
    native.check(native.lib().emmy_device_init(0))
    kw = {}
    for item in filter(None, (args.size or "").split(",")):
        key, val = item.split("=")
        kw[key] = float(val) if "." in val or "e-" in val else int(val)
    print(json.dumps(measure_case(args.case, kw, args.steps, args.warmup,
                                  extras=args.case == "vector_add")), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--case", default=None, help="time one synthesised configuration")
    ap.add_argument("--size", default=None, help="size overrides for --case, k=v,k=v")
    ap.add_argument("--no-categories", action="store_true",
                    help="skip the per-category kernels after the headline workload")
    ap.add_argument("--problems", action="store_true",
                    help="time the reference's 15 open problems, ours and the reference PTX")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.case:
        run_case(args)
        return
    if args.problems:
        run_problems(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    from emmy_b200 import dist as D
    if world > 1:
        import torch
        torch.cuda.set_device(local)
        D.init("nccl", D.from_env(), timeout_s=120, device=torch.device("cuda", local))
    try:
        run_ours(args, rank, world, local)
    finally:
        D.finish()


if __name__ == "__main__":
    main()

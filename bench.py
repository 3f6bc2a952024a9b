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
            "config": {"workload": WORKLOAD, "step": "one pass of the three reductions"},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads,
                             "kind": "port",
                             "sample": "full workload (3 GiB read), numpy reductions split "
                                       f"over {threads} threads"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# GPU path
# --------------------------------------------------------------------------

def run_ours(args, rank: int, world: int, local: int) -> None:
    import numpy as np
    import torch
    from emmy_b200 import dist as D
    from emmy_b200 import harness, native

    torch.cuda.set_device(local)
    native.check(native.lib().emmy_device_init(local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream

    probs = make_problems()
    kerns = {n: harness.CompiledKernel(*p.build()) for n, p in probs}
    nbytes = {n: bytes_of(p) for n, p in probs}
    step_bytes = sum(nbytes.values())

    x_sum_h, x_rows_h = host_inputs(rank)
    x_sum_h, x_rows_h = x_sum_h.pin_memory(), x_rows_h.pin_memory()
    x_sum = x_sum_h.to(dev)
    x_rows = x_rows_h.to(dev)
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

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # correctness spot check of this rank's results (cheap, outside timing)
    ref_sum = float(x_sum.double().sum())
    if world == 1:
        assert abs(float(out_sum) - ref_sum) <= 1e-4 * abs(ref_sum), (float(out_sum), ref_sum)
    ref_rs = x_rows.double().sum(-1)
    assert torch.allclose(out_rs.double(), ref_rs, rtol=1e-4, atol=1e-4 * float(ref_rs.abs().max()))

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

    # e2e through the C ABI with host buffers: copies in, launch, result out
    host_out = {"full_sum": np.zeros(1, np.float32), "row_sum": np.zeros(32768, np.float32),
                "row_mean": np.zeros(32768, np.float32)}
    x_sum_np, x_rows_np = x_sum_h.numpy(), x_rows_h.numpy()
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
    e2e_steps = max(1, min(args.steps, 5))
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
    # the host outputs of the end-to-end path are right (row kernels on the
    # input the step copied once), checked on a few rows outside the timing
    chk = x_rows_np[:16].astype(np.float64)
    assert np.allclose(host_out["row_sum"][:16], chk.sum(1), rtol=1e-4, atol=1e-3)
    assert np.allclose(host_out["row_mean"][:16], chk.mean(1), rtol=1e-4, atol=1e-4)

    # reference compiler's PTX for the same IRs, JIT-run on this GPU
    ref_ptx = {}
    for n in order:
        f = REPO / "oracle" / "_ref" / f"{n}.ptx"
        if not f.exists():
            continue
        img = native.Image(f.read_text())
        mod = native.Module(img.data)
        kh = mod.kernel("ref_" + kerns[n].entry)
        k = kerns[n]
        arr, keep = k.params(ptrs[n])
        zero = [(out_sum.data_ptr(), 4)] if n == "full_sum" else []
        from emmy_b200 import harness as H  # noqa: F401
        import ctypes
        it = 10
        outbuf = (ctypes.c_float * it)()
        zd = (ctypes.c_uint64 * 1)(*([z[0] for z in zero] or [0]))
        zb = (ctypes.c_size_t * 1)(*([z[1] for z in zero] or [0]))
        native.check(L.emmy_time_launches(kh.h, native.u32x3(k.grid), native.u32x3(k.block),
                                          k.smem, None, arr, sh, 2, it, 0, 0, zd, zb,
                                          len(zero), outbuf))
        ref_ptx[n] = statistics.median(list(outbuf))
    # our kernels under the same protocol as the reference PTX (median of 10)
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
    cpu = None
    if rank == 0 and world == 1:
        xs, xr = x_sum_np, x_rows_np
        cpu_reductions(xs, xr, 1)
        ts = [cpu_reductions(xs, xr, 1) for _ in range(3)]
        sec = statistics.median(ts)
        cpu = {"value": round(step_bytes / sec / 1e9, 3), "unit": "GB/s", "cores": 1,
               "kind": "port",
               "sample": "full workload once per run (median of 3), numpy float32 reductions "
                         "as the reference's refs.py, single thread"}
    categories = None
    if world == 1 and not args.no_categories:
        # every other category's kernel at its BASELINE size (own buffers;
        # the reductions inputs are released first)
        del x_sum, x_rows, devt, host, ptrs, params
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        categories = {}
        for nm in CATEGORY_CASES:
            try:
                # 10 launches as a burst, comparable with the burst peaks (longer
                # runs of the contractions settle at the power-capped clock); the
                # microsecond-scale vector add takes 50 for a stable median
                r = measure_case(nm, {}, 50 if nm == "vector_add" else 10, 3)
            except Exception as e:  # report, keep the headline line
                categories[nm] = {"error": f"{type(e).__name__}: {e}"[:200]}
                continue
            categories[nm] = {kk: r[kk] for kk in ("template", "ms_median", "GB/s", "TFLOP/s",
                                                   "frac", "reference_ptx_ms",
                                                   "speedup_vs_reference_ptx") if kk in r}
    shards = None
    if world > 1 and not args.no_categories:
        # the configurations that shard without an exchange, strong scaling:
        # each rank times its shard of the BASELINE problem; the job's time
        # is the max over ranks
        del x_sum, x_rows, devt, host, ptrs, params
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        from emmy_b200 import synth
        shards = {}
        for nm in D.SHARDED:
            kw = D.shard_kwargs(nm, rank, world)
            try:
                r = measure_case(nm, kw, 10, 3)
                ms_r, err = r["ms_median"], None
            except Exception as e:  # every rank still joins the max below
                ms_r, err = float("inf"), f"{type(e).__name__}: {e}"[:200]
            ms_all = D.max_over_ranks(ms_r, device=dev)
            full = synth.config(nm)
            flops = synth.algorithmic_flops(full)
            shards[nm] = {"partition": D.SHARDED[nm][0], "rank0_shard": D.shard_kwargs(nm, 0, world),
                          "ms_max_over_ranks": round(ms_all, 5),
                          "TFLOP/s": round(flops / (ms_all / 1e3) / 1e12, 1) if ms_all < 1e30 else None,
                          "scaling": "strong"}
            if err:
                shards[nm]["error"] = err
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (torch.Generator seeds 1000*rank+{0,1}; BASELINE distributions)",
            "config": {"workload": WORKLOAD, "per_rank_bytes_per_step": step_bytes,
                       "l2": "each input is 1 GiB > 126 MB L2; no flush needed",
                       "parallelism": f"weak scaling over {world} rank(s); full sum "
                                      "finished by NCCL all-reduce"},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                         "peak": hbm, "peak_source": src, "unit": "GB/s",
                         "frac": round(achieved / hbm, 3), "traffic": traffic,
                         "algorithmic_bytes": nbytes[dom]},
            "kernels": cats,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "path": "emmy_run_host (C ABI) from pinned host memory"},
            "gpu_launches": 3 * args.steps,
            "clocks": clk.summary(),
            "categories": categories,
            "shards": shards,
        }
        print(json.dumps(line), flush=True)


def measure_case(name: str, kw: dict, steps: int, warmup: int) -> dict:
    """Time one synthesised configuration: ``steps`` launches through the C ABI,
    each bracketed by CUDA events on the launching stream; L2 flushed between
    launches when the inputs would fit in it.  Includes the reference
    compiler's PTX for the same IR (``oracle/_ref``) when it exists."""
    import numpy as np
    import torch

    from emmy_b200 import harness, native, synth

    p = synth.config(name, **kw)
    g, m = p.build()
    kern = harness.CompiledKernel(g, m)
    bufs = harness.Buffers.random(kern, seed=0)
    stream = torch.cuda.current_stream().cuda_stream
    in_bytes = sum(t.numel() * t.element_size() for n, t in bufs.t.items()
                   if not bufs.args[n].get("output"))
    flush = fb = None
    if in_bytes < 2 * 126 * 2 ** 20:
        fb = torch.empty(512 * 2 ** 20, dtype=torch.uint8, device="cuda")
        flush = (fb.data_ptr(), fb.numel())
    ms = kern.time(bufs.ptrs(), warmup=warmup, iters=steps, stream=stream,
                   flush=flush, zero=bufs.zero_list())
    med = float(np.median(ms))
    hbm, src = peaks()
    nb = synth.algorithmic_bytes(p)
    flops = synth.algorithmic_flops(p)
    line = {"case": name, "size": kw, "template": kern.kind, "entry": kern.entry,
            "ms_median": round(med, 5), "ms_min": round(float(np.min(ms)), 5),
            "launches": steps, "l2_flush": flush is not None,
            "regs": kern.image.registers().get(kern.entry)}
    if flops:
        tf = flops / (med / 1e3) / 1e12
        mp = REPO / "MEASURED_PEAKS.json"
        peak = float(json.loads(mp.read_text())["bf16_tflops"]) if mp.exists() else 1590.0
        basis = "measured bf16 peak"
        if kern.kind == "gemm" and getattr(kern.compiler.template, "mode", "") == "tf32x3":
            # fp32 through 3xTF32: tf32 runs at half the bf16 rate and every
            # product costs three tf32 MMAs
            peak, basis = peak / 2 / 3, "3xTF32 effective = measured bf16 peak / 2 / 3"
        line.update({"TFLOP/s": round(tf, 1), "peak": round(peak, 1), "peak_basis": basis,
                     "frac": round(tf / peak, 3), "flops": flops})
    else:
        gbs = nb / (med / 1e3) / 1e9
        line.update({"GB/s": round(gbs, 1), "peak": hbm, "peak_source": src,
                     "frac": round(gbs / hbm, 3), "algorithmic_bytes": nb})
    f = REPO / "oracle" / "_ref" / f"{name}.ptx"
    if f.exists() and not kw:
        # the reference compiler's PTX for the same IR, launched under the same
        # meta entry from its own text (its parameters are the meta arguments
        # alone: no tensor maps, no cluster)
        ref = harness.CompiledKernel.from_ptx(f.read_text(),
                                              dict(kern.info, entry="ref_" + kern.entry))
        rms = ref.time(bufs.ptrs(), warmup=2, iters=min(steps, 10), stream=stream,
                       flush=flush, zero=bufs.zero_list())
        line["reference_ptx_ms"] = round(float(np.median(rms)), 5)
        line["speedup_vs_reference_ptx"] = round(float(np.median(rms)) / med, 2)
        ref._module.unload()
    del bufs, fb
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return line


CATEGORY_CASES = ["vector_add", "vector_add_large", "rmsnorm", "softmax", "l2norm", "matmul_bf16", "matmul_f32",
                  "attention", "attention_d64"]


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
    print(json.dumps(measure_case(args.case, kw, args.steps, args.warmup)), flush=True)


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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.case:
        run_case(args)
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

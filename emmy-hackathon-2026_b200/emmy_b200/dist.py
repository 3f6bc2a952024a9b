"""Multi-GPU plumbing: one process per GPU, torch.distributed for the exchange.

The kernels of this path are independent per row / per output tile / per
element chunk, so a multi-GPU run is the same single-GPU kernels on shards.
The only cross-GPU reduction of the path is the global sum: each rank's
kernel produces a partial ``f32[1]`` and :func:`global_sum` finishes it with
one all-reduce (NCCL over NVLink/NVSwitch on GPUs; gloo in the CPU tests).

Two ways of sharding a configuration:

* weak scaling (the benchmark): every rank owns a full-size shard of each
  input, drawn with its own seed (:func:`rank_seed`), so per-GPU work is fixed
  as the number of GPUs grows;
* strong scaling: a fixed global shape split into contiguous row / element
  ranges (:func:`shard_range`).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Rank:
    rank: int
    world: int
    local: int

    @property
    def is_root(self) -> bool:
        return self.rank == 0


def from_env() -> Rank:
    """RANK / WORLD_SIZE / LOCAL_RANK as torchrun sets them (1 process if unset)."""
    return Rank(int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
                int(os.environ.get("LOCAL_RANK", 0)))


def init(backend: str, r: Rank, timeout_s: float = 120.0, device=None) -> None:
    """Initialise the process group (short timeout: a rank that never joins or
    dies ends the others' next collective with an error instead of a hang)."""
    import torch.distributed as dist
    if r.world <= 1 or dist.is_initialized():
        return
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)


def finish() -> None:
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()


def rank_seed(base: int, rank: int) -> int:
    """Seed of a rank's shard of an input whose single-GPU seed is ``base``
    (rank 0 keeps the single-GPU seed)."""
    return base + 1000 * rank


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, end) of ``n`` units for ``rank``; the first ``n % world``
    ranks get one extra unit."""
    q, r = divmod(n, world)
    start = rank * q + min(rank, r)
    return start, start + q + (1 if rank < r else 0)


# the configurations measured at N > 1 as strong scaling of the BASELINE
# problem: (partition, number of units, unit size).  Rows for the row
# reductions and fused row ops, 2048-element chunks for the pointwise add,
# 256-row bands of A and C for matmul (B replicated), (batch, head) pairs for
# attention -- none of them exchanges data -- and for the full sum whole CTA
# slices (131,072 elements each, one CTA of the one-GPU launch; a shard of
# fewer than 4096 slices runs each on 2, 4, ... CTAs), whose per-rank
# partial sums are finished by one all-reduce.  (The 8-GPU shard, 2^25
# elements: 25.0 us a step at 1024 CTAs, 23.0 at 4096, one GPU, graph replays.)
SUM_SLICE = 268_435_456 // 2048
SUM_MIN_CTAS = 4096
SHARDED = {
    "vector_add": ("elements", 1_048_576 // 2048, 2048),
    "full_sum": ("slices", 2048, SUM_SLICE),
    "row_sum": ("rows", 32768, 1), "row_mean": ("rows", 32768, 1),
    "rmsnorm": ("rows", 65536, 1), "softmax": ("rows", 65536, 1), "l2norm": ("rows", 65536, 1),
    "matmul_bf16": ("M", 16384 // 256, 256), "matmul_f32": ("M", 16384 // 256, 256),
    "attention": ("heads", 8 * 32, 1), "attention_d64": ("heads", 8 * 32, 1),
}


def shard_kwargs(name: str, rank: int, world: int) -> dict:
    """Size overrides of ``synth.config(name)`` for ``rank``'s shard of the
    BASELINE problem (strong scaling: the shards of all ranks together are
    the single-GPU problem): a contiguous range of the configuration's units
    (``SHARDED``).  Attention shards are synthesised as B=1, H=pairs."""
    dim, total, unit = SHARDED[name]
    lo, hi = shard_range(total, rank, world)
    k = hi - lo
    if dim == "rows":
        return {"rows": k}
    if dim == "elements":
        return {"n": k * unit}
    if dim == "slices":
        # a shard of few slices splits each over several CTAs (a power of
        # two, so the slice divides evenly), keeping at least SUM_MIN_CTAS
        # CTAs in the launch: 256 one-slice CTAs on 148 SMs leave HBM idle
        split = 1 << max(0, (SUM_MIN_CTAS // max(k, 1)).bit_length() - 1)
        return {"n": k * unit, "ctas": k * split}
    if dim == "M":
        return {"M": k * unit}
    return {"B": 1, "H": k}


def shard_offset(name: str, rank: int, world: int) -> int:
    """Index of ``rank``'s first row / element / (batch, head) pair in the
    BASELINE problem."""
    _, total, unit = SHARDED[name]
    return shard_range(total, rank, world)[0] * unit


def global_sum(partial) -> None:
    """In-place all-reduce (sum) of each rank's partial result."""
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(partial)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of a per-rank scalar (timings are reported as the max)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()

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


# the configurations whose work shards across GPUs without an exchange, with
# their BASELINE sizes: matmul by 256-row bands of A and C (B replicated),
# attention by (batch, head) pairs
SHARDED = {"matmul_bf16": ("M", 16384, 256), "matmul_f32": ("M", 16384, 256),
           "attention": ("heads", 8 * 32, 1), "attention_d64": ("heads", 8 * 32, 1)}


def shard_kwargs(name: str, rank: int, world: int) -> dict:
    """Size overrides of ``synth.config(name)`` for ``rank``'s shard of the
    BASELINE problem (strong scaling: the shards of all ranks together are
    the single-GPU problem).  Matmul: a contiguous range of 256-row bands
    (the CTA-pair tiles' rows); attention: a contiguous range of the
    B x H = 256 (batch, head) pairs, synthesised as B=1, H=count."""
    dim, total, unit = SHARDED[name]
    lo, hi = shard_range(total // unit, rank, world)
    if dim == "M":
        return {"M": (hi - lo) * unit}
    return {"B": 1, "H": hi - lo}


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

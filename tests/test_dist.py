"""The multi-rank host logic on CPU: two gloo ranks, each reducing its own
shard, finished by the all-reduce (the global-sum exchange of the path);
max-over-ranks timing; shard ranges; and a rank that never joins makes the
other's collective fail inside the process-group timeout instead of
hanging."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from emmy_b200 import dist as D


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import torch
    r = D.from_env()
    D.init("gloo", r, timeout_s=30)
    n = 1 << 16
    lo, hi = D.shard_range(n, r.rank, r.world)
    x = np.random.default_rng(D.rank_seed(0, 0)).uniform(0, 1, n).astype(np.float32)
    part = torch.tensor([x[lo:hi].astype(np.float64).sum()], dtype=torch.float64)
    D.global_sum(part)
    mx = D.max_over_ranks(float(rank + 1))
    q.put((rank, float(part), mx, float(x.astype(np.float64).sum())))
    D.barrier()
    D.finish()


def test_two_rank_global_sum():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, total, mx, ref in res:
        assert abs(total - ref) <= 1e-9 * ref
        assert mx == 2.0


def _lonely(port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0"})
    try:
        D.init("gloo", D.from_env(), timeout_s=3)
        q.put("joined")
    except Exception as e:  # the peer never joins: rendezvous times out
        q.put(type(e).__name__)


def test_missing_rank_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_port(), q))
    p.start()
    out = q.get(timeout=120)
    p.join(timeout=60)
    assert out != "joined"


@pytest.mark.parametrize("n,world", [(10, 3), (32768, 8), (5, 8), (0, 2)])
def test_shard_ranges_cover(n, world):
    seen = []
    for r in range(world):
        a, b = D.shard_range(n, r, world)
        seen.extend(range(a, b))
    assert seen == list(range(n))


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_kwargs_cover_the_problem(world):
    """The per-rank shards of every strong-scaled configuration add up to the
    BASELINE problem, back to back from each rank's offset, and every shard's
    IR is one the templates accept (rows, pointwise, tensor-core kernels)."""
    from emmy_b200 import synth
    from emmy_b200.compiler import compile_graph
    size = {"vector_add": ("n", 1_048_576), "full_sum": ("n", 268_435_456),
            "row_sum": ("rows", 32768), "row_mean": ("rows", 32768), "rmsnorm": ("rows", 65536),
            "softmax": ("rows", 65536), "l2norm": ("rows", 65536), "matmul_bf16": ("M", 16384),
            "matmul_f32": ("M", 16384), "attention": ("H", 256), "attention_d64": ("H", 256)}
    assert set(size) == set(D.SHARDED)
    for name, (key, total) in size.items():
        parts = [D.shard_kwargs(name, r, world) for r in range(world)]
        offs = [D.shard_offset(name, r, world) for r in range(world)]
        assert sum(p[key] for p in parts) == total
        assert offs == [sum(p[key] for p in parts[:r]) for r in range(world)]
        if name.startswith("matmul"):
            assert all(p["M"] % 256 == 0 for p in parts)
        if name == "full_sum":
            # whole slices per rank, each on a power-of-two number of CTAs,
            # at least 1024 CTAs a launch (2048 slices: one CTA each at N=1)
            for p in parts:
                split = p["ctas"] * D.SUM_SLICE // p["n"]
                assert p["n"] % D.SUM_SLICE == 0 and split & (split - 1) == 0
                assert p["ctas"] >= min(D.SUM_MIN_CTAS, p["n"] // D.SUM_SLICE)
                assert D.SUM_SLICE % split == 0 and p["ctas"] < 2 * D.SUM_MIN_CTAS or split == 1
    want = {"vector_add": "pointwise", "full_sum": "rows", "row_mean": "rows", "softmax": "rows",
            "matmul_bf16": "gemm", "attention_d64": "attention"}
    for name, kind in want.items():
        kw = D.shard_kwargs(name, world - 1, world)
        g, m = synth.config(name, **kw).build()
        assert compile_graph(g, m).kind == kind, name


def _handles(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    from emmy_b200 import peer
    D.init("gloo", D.from_env(), timeout_s=30)
    got = peer.exchange_handles(bytes([rank + 1]) * 64, world)
    q.put((rank, got))
    D.barrier()
    D.finish()


def test_peer_handles_are_exchanged_in_rank_order():
    """The NVLink finish of the global sum (``peer.PeerSum``) maps every
    rank's slot array from the 64-byte handles the ranks exchange through the
    process group: each rank receives all of them, in rank order (gloo, two
    ranks on CPU; the mapping itself needs GPUs)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_handles, args=(r, 3, port, q)) for r in range(3)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got in res:
        assert got == [bytes([r + 1]) * 64 for r in range(3)]


def test_peer_sum_kernel_assembles_and_checks(native_lib):
    """The peer-sum kernel assembles for sm_100a and passes the static PTX
    checks; every poll is bounded by %globaltimer and reports code 9."""
    from emmy_b200 import native, peer, ptxcheck
    img = native.Image(peer.PEER_SUM_PTX)
    assert img.registers().get("emmy_peer_sum")
    assert ptxcheck.check(peer.PEER_SUM_PTX) == []
    assert "%globaltimer" in peer.PEER_SUM_PTX and f"], {peer.STATUS_TIMEOUT};" in peer.PEER_SUM_PTX
    assert "multimem" not in peer.PEER_SUM_PTX and "multicast" not in peer.PEER_SUM_PTX

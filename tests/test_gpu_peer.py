"""The NVLink finish of the global sum (``peer.PeerSum``) on two GPUs: one
process per GPU, each rank's partial written into every rank's slot over
peer memory, summed in rank order on every rank.  Needs two GPUs (skipped
otherwise: ranks whose kernels wait on one another never share a GPU)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "NCCL_NVLS_ENABLE": "0"})
    import torch
    from emmy_b200 import dist as D
    from emmy_b200 import native, peer
    torch.cuda.set_device(rank)
    native.check(native.lib().emmy_device_init(rank))
    D.init("gloo", D.from_env(), timeout_s=60)
    ps = peer.PeerSum(rank, world)
    vals = np.random.default_rng(5).uniform(-1, 1, (6, world)).astype(np.float32)
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    got = []
    for i in range(4):                      # eager launches: epochs 1..4
        out.fill_(float(vals[i, rank]))
        ps.launch(out.data_ptr(), stream)
        got.append(float(out.item()))
    # a CUDA graph of fill + finish, replayed (epochs 5, 6 from device memory)
    g = torch.cuda.CUDAGraph()
    src = torch.tensor([float(vals[4, rank])], device="cuda")
    torch.cuda.synchronize()
    D.barrier()
    with torch.cuda.graph(g):
        out.copy_(src)
        ps.launch(out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    for i in (4, 5):
        src.fill_(float(vals[i, rank]))
        g.replay()
        torch.cuda.synchronize()
        got.append(float(out.item()))
    del g
    status = ps.status()
    D.barrier()
    ps.close(barrier=D.barrier)
    q.put((rank, got, status))
    D.barrier()
    D.finish()


def test_peer_sum_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    vals = np.random.default_rng(5).uniform(-1, 1, (6, world)).astype(np.float32)
    want = []
    for i in range(6):                      # rank order, f32 adds from 0, as the kernel
        acc = np.float32(0)
        for r in range(world):
            acc = np.float32(acc + vals[i, r])
        want.append(float(acc))
    for rank, got, status in res:
        assert status == 0
        assert got == want, (rank, got, want)


# ---------------------------------------------------------------------------
# the fused form: the split full-sum kernel's last CTA runs the exchange
# ---------------------------------------------------------------------------

def _fused_run(rank, world, n_per_rank=1 << 20, ctas=64, reps=3):
    """Compile the split full sum with ``peer_finish``, launch it ``reps``
    times eagerly and twice from a CUDA graph on this rank's slice; returns
    (sums read back after each launch, the float64 sum of this rank's slice,
    the module's status word)."""
    import torch
    from emmy_b200 import harness, native, peer, synth
    g, m = synth.config("full_sum", n=n_per_rank, ctas=ctas).build()
    m["kernels"][0]["peer_finish"] = True
    kern = harness.CompiledKernel(g, m)
    assert kern.peer_params == [n for n, _ in peer.FUSED_PARAMS]
    bufs = harness.Buffers.random(kern, seed=rank)
    ps = peer.PeerSum(rank, world)
    ptrs = bufs.ptrs()
    ptrs.update(ps.fused_values())
    out = bufs.t["sum_1"]
    stream = torch.cuda.current_stream().cuda_stream
    got = []
    for _ in range(reps):
        out.zero_()
        kern.launch(ptrs, stream)
        torch.cuda.synchronize()
        got.append(float(out.item()))
    g_ = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_):
        out.zero_()
        kern.launch(ptrs, torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        g_.replay()
        torch.cuda.synchronize()
        got.append(float(out.item()))
    del g_
    import ctypes
    addr, _ = kern.module().global_addr("__emmy_status")
    st = ctypes.c_uint32()
    native.check(native.lib().emmy_memcpy_dtoh_async(ctypes.addressof(st), addr, 4, None))
    native.check(native.lib().emmy_stream_sync(None))
    part = float(np.sum(bufs.t["x"].cpu().numpy(), dtype=np.float64))
    return got, part, st.value, ps


def test_fused_sum_finish_one_gpu():
    """One rank: the sum kernel's last CTA finishes the sum with itself --
    the completion counter finds exactly one last CTA per launch and resets
    for the next (five launches, two of them graph replays), the epoch
    advances from device memory, status 0, the sum within rel 1e-4 of the
    float64 sum."""
    import torch
    from emmy_b200 import native
    torch.cuda.set_device(0)
    native.check(native.lib().emmy_device_init(0))
    got, want, status, ps = _fused_run(0, 1)
    ps.close()
    assert status == 0
    for v in got:
        assert abs(v - want) <= 1e-4 * abs(want), (v, want)


def _fused_rank(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "NCCL_NVLS_ENABLE": "0"})
    import torch
    from emmy_b200 import dist as D
    from emmy_b200 import native
    torch.cuda.set_device(rank)
    native.check(native.lib().emmy_device_init(rank))
    D.init("gloo", D.from_env(), timeout_s=60)
    D.barrier()
    got, part, status, ps = _fused_run(rank, world)
    D.barrier()
    ps.close(barrier=D.barrier)
    q.put((rank, got, part, status))
    D.barrier()
    D.finish()


def test_fused_sum_finish_two_gpus():
    """Two ranks, one process per GPU: every launch of the fused kernel
    leaves the same bits on both ranks, the sum of both ranks' slices
    (within rel 1e-4 of the float64 sum), status 0."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_fused_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = sum(part for _, _, part, _ in res)
    assert res[0][1] == res[1][1]
    for rank, got, part, status in res:
        assert status == 0
        for v in got:
            assert abs(v - want) <= 1e-4 * abs(want), (rank, v, want)

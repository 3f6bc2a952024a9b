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

"""The one entry point that allocates nothing, ``emmy_rmsnorm_noalloc``, on
the GPU, called through the C ABI.

It exists for callers that cannot allocate device memory when they call into
the library (an allocator that owns all device memory, code running while a
CUDA graph is being built, a fixed memory budget): it runs the two-kernel
RMSNorm with the per-row intermediate held in a static device array instead of
a buffer the caller allocates.  Its output must match the existing path -- the
same two kernels launched with ``emmy_launch`` and a caller-allocated
intermediate -- within the RMSNorm tolerance used by the other tests, on two
calls in a row with different inputs (the second call reuses the array the
first one filled), and the CPU oracle within the same tolerance.  A row count
the array cannot hold, or launches that do not match the row count (a first
grid wider than the array, a second grid that misses elements), must be
refused with EMMY_EINVAL and a message before anything runs.

This file is collected last, so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROWS, COLS = 1024, 2048
RTOL, ATOL = 1e-5, 1e-5


def _setup():
    import torch
    from emmy_b200 import harness, native, synth
    irs, meta = synth.rmsnorm_two_kernel(rows=ROWS, cols=COLS).build()
    k1, k2 = (harness.CompiledKernel(irs[k["entry"]], meta) for k in meta["kernels"])
    assert (k1.entry, k2.entry) == ("k_rms_meansq", "k_rms_apply")
    consts = {}
    for k in meta["kernels"]:
        for a in k["args"]:
            if "data" in a:
                consts[a["name"]] = torch.tensor(a["data"], dtype=torch.float32, device="cuda")
    return native, k1, k2, consts


def _existing_path(k1, k2, consts, x, w):
    """The two kernels through emmy_launch, intermediate allocated by the caller."""
    import torch
    ms = torch.empty(ROWS, dtype=torch.float32, device="cuda")
    y = torch.zeros(ROWS * COLS, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    k1.launch({"mean_count": consts["mean_count"].data_ptr(), "x": x.data_ptr(),
               "ms": ms.data_ptr()}, s)
    k2.launch({"add_c1": consts["add_c1"].data_ptr(), "x": x.data_ptr(), "ms": ms.data_ptr(),
               "w": w.data_ptr(), "mul_1": y.data_ptr()}, s)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _noalloc(native, k1, k2, consts, x, w, y, rows=ROWS, cols=COLS, grid1=None, grid2=None):
    import torch
    from emmy_b200.native import u32x3
    rc = native.lib().emmy_rmsnorm_noalloc(
        k1.kernel().h, u32x3(grid1 or k1.grid), u32x3(k1.block),
        k2.kernel().h, u32x3(grid2 or k2.grid), u32x3(k2.block),
        consts["mean_count"].data_ptr(), consts["add_c1"].data_ptr(), x.data_ptr(),
        w.data_ptr(), y.data_ptr(), rows, cols,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return rc


def test_noalloc_matches_existing_path_on_two_calls():
    import torch
    native, k1, k2, consts = _setup()
    w = torch.empty(COLS, device="cuda").uniform_(0.5, 1.5)
    y = torch.zeros(ROWS * COLS, dtype=torch.float32, device="cuda")
    for seed in (0, 1):
        g = torch.Generator(device="cuda").manual_seed(seed)
        x = torch.randn(ROWS * COLS, device="cuda", generator=g) * (1 + 3 * seed)
        ref = _existing_path(k1, k2, consts, x, w)
        y.zero_()
        assert _noalloc(native, k1, k2, consts, x, w, y) == 0, native.lib().emmy_last_error()
        got = y.cpu().numpy()
        assert np.allclose(got, ref, rtol=RTOL, atol=ATOL), float(np.max(np.abs(got - ref)))
        # and the CPU oracle of RMSNorm on the same inputs
        from oracle import expr
        want = expr.rmsnorm(x.cpu().numpy().reshape(ROWS, COLS), w.cpu().numpy(),
                            float(consts["add_c1"].cpu()[0]))
        assert np.allclose(got.reshape(ROWS, COLS), want, rtol=RTOL, atol=ATOL), \
            float(np.max(np.abs(got.reshape(ROWS, COLS) - want)))


def _refused(native, k1, k2, consts, match, **kw):
    import torch
    x = torch.zeros(ROWS * COLS, device="cuda")
    w = torch.ones(COLS, device="cuda")
    y = torch.full((ROWS * COLS,), 7.0, device="cuda")
    rc = _noalloc(native, k1, k2, consts, x, w, y, **kw)
    assert rc == -1                                   # EMMY_EINVAL
    assert match in native.lib().emmy_last_error()
    assert torch.all(y == 7.0)                        # nothing ran


def test_noalloc_rejects_oversize():
    native, k1, k2, consts = _setup()
    _refused(native, k1, k2, consts, b"scratch array holds", rows=65536 + 1)


def test_noalloc_rejects_launches_that_do_not_match_rows():
    """The kernels write and read one entry per row of their launch: a first
    grid wider than the array (here with a small row count) or a second grid
    that does not cover rows x cols elements is refused before any launch."""
    native, k1, k2, consts = _setup()
    _refused(native, k1, k2, consts, b"grid1", grid1=(65536 + 4096, 1, 1))
    _refused(native, k1, k2, consts, b"grid1", grid1=(ROWS, 2, 1))
    g2 = k2.grid[0]
    _refused(native, k1, k2, consts, b"grid2", grid2=(g2 - 1, 1, 1))
    _refused(native, k1, k2, consts, b"grid2", grid2=(g2 + 1, 1, 1))
    _refused(native, k1, k2, consts, b"grid2", cols=COLS * 2)

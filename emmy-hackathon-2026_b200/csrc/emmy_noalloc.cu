// emmy_noalloc.cu -- the one entry point of this library that allocates nothing.
//
// Some callers cannot allocate device memory when they call us: an allocator
// that owns all device memory and forbids cudaMalloc from inside (a
// framework's caching allocator or a pool sized at start-up), code running
// while a CUDA graph is being built, or a host program whose memory budget is
// fixed before it runs.  The two-kernel RMSNorm (the row mean of squares
// written to an intermediate, then y = x * rsqrt(ms + eps) * w) needs one
// float of scratch per row between its kernels; every other path of this
// library takes that buffer from the caller.  emmy_rmsnorm_noalloc keeps it
// in a file-scope device array instead, so the caller passes only inputs and
// outputs.
//
// The price: the array (EMMY_NOALLOC_MAX_ROWS floats, 256 KiB) is held by every
// GPU that loads this library until the process exits; calls may use at most
// that many rows; and every call shares it, so calls that overlap on the GPU
// (two streams, two threads) race on it.  The first call on a device loads
// this file's device code there, which is when the array is reserved on that
// device: a caller with a fixed memory budget makes that first call at
// start-up.
//
// The row count is checked against the launches, not only against the
// caller's word: the first kernel writes one entry per CTA of its grid, so
// grid1 must be (rows, 1, 1); the second reads the entry of each element's
// row, one thread per element, so its one-dimensional grid2 x block2 must
// cover rows x cols elements and no whole block more.  Kernels compiled for
// other shapes than (rows, cols) are outside what these checks can see: pass
// the pair compiled from the two IRs for exactly these rows and columns.
#include "../../include/emmy_b200.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

int emmy_internal_fail(int code, const char *msg);   // emmy_runtime.cpp

// The row scratch.  Host code must not pass this name to a kernel: on the host
// it is a stand-in symbol, not a device address -- the address comes from
// cudaGetSymbolAddress below, once per device.
static __device__ __align__(256) float g_rows_scratch[EMMY_NOALLOC_MAX_ROWS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
uint64_t g_scratch_addr[kMaxDevices];   // 0 until set up on that device

int fail_msg(int code, const char *fmt, const char *a, long b = 0, long c = 0) {
  char buf[512];
  snprintf(buf, sizeof buf, fmt, a, b, c);
  return emmy_internal_fail(code, buf);
}

// Device address of the scratch array on the current device.  The first call
// on a device resolves it (cudaGetSymbolAddress with that device current),
// later calls reuse the cached address.
int scratch_on_current_device(uint64_t *out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail_msg(EMMY_ENODRIVER, "emmy_rmsnorm_noalloc: cudaGetDevice failed: %s",
                    cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail_msg(EMMY_EINVAL, "emmy_rmsnorm_noalloc: %s device %ld", "unsupported", dev);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_rows_scratch);
    if (e != cudaSuccess || !p) {
      // the device code is built for sm_100a only: name the device's
      // architecture, the usual reason for "no kernel image"
      int major = 0, minor = 0;
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
      return fail_msg(EMMY_ENODRIVER,
                      "emmy_rmsnorm_noalloc: cudaGetSymbolAddress failed (%s); this library's "
                      "device code is built for sm_100a, device is sm_%ld%ld",
                      cudaGetErrorString(e), major, minor);
    }
    g_scratch_addr[dev] = reinterpret_cast<uint64_t>(p);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace

extern "C" EMMY_API int emmy_rmsnorm_noalloc(
    emmy_kernel_t meansq, const uint32_t grid1[3], const uint32_t block1[3],
    emmy_kernel_t apply, const uint32_t grid2[3], const uint32_t block2[3],
    uint64_t mean_count, uint64_t add_c1, uint64_t x, uint64_t w, uint64_t y,
    int rows, int cols, void *stream) {
  if (!meansq || !apply || !grid1 || !block1 || !grid2 || !block2 || !mean_count || !add_c1 ||
      !x || !w || !y)
    return emmy_internal_fail(EMMY_EINVAL, "emmy_rmsnorm_noalloc: bad argument");
  if (rows <= 0 || rows > EMMY_NOALLOC_MAX_ROWS)
    return fail_msg(EMMY_EINVAL,
                    "emmy_rmsnorm_noalloc: %s %ld rows, the scratch array holds 1..%ld",
                    "cannot take", rows, static_cast<long>(EMMY_NOALLOC_MAX_ROWS));
  if (cols <= 0)
    return fail_msg(EMMY_EINVAL, "emmy_rmsnorm_noalloc: %s %ld columns", "cannot take", cols);
  // the launches must be the ones the row count describes (checked in 64 bits:
  // a grid of three 32-bit extents overflows 32)
  const uint64_t g1 = uint64_t(grid1[0]) * grid1[1] * grid1[2];
  if (grid1[1] != 1 || grid1[2] != 1 || g1 != uint64_t(rows))
    return fail_msg(EMMY_EINVAL,
                    "emmy_rmsnorm_noalloc: %s grid1 of %ld CTAs for %ld rows (one CTA per row)",
                    "refusing", static_cast<long>(g1 > 0x7fffffffull ? 0x7fffffffull : g1), rows);
  // the element kernel's launch is one-dimensional (at most 2^31 x 1024 threads)
  const uint64_t t2 = block2[0], g2 = grid2[0];
  const uint64_t cells = uint64_t(rows) * uint64_t(cols);
  if (grid2[1] != 1 || grid2[2] != 1 || block2[1] != 1 || block2[2] != 1 || t2 == 0 ||
      t2 > 1024 || g2 * t2 < cells || g2 * t2 >= cells + t2)
    return fail_msg(EMMY_EINVAL,
                    "emmy_rmsnorm_noalloc: %s grid2 x block2 of %ld threads for %ld elements "
                    "(one thread per element)", "refusing",
                    static_cast<long>(g2 * t2 > 0x7fffffffull ? 0x7fffffffull : g2 * t2),
                    static_cast<long>(cells > 0x7fffffffull ? 0x7fffffffull : cells));
  uint64_t ms = 0;
  if (int e = scratch_on_current_device(&ms)) return e;
  // The first kernel writes every row's entry before the second reads it, so
  // nothing left from an earlier call can leak into this one and the array
  // needs no clearing.  Parameters follow the kernels' meta arg_order.
  void *p1[] = {&mean_count, &x, &ms};
  if (int e = emmy_launch(meansq, grid1, block1, 0, nullptr, p1, stream)) return e;
  void *p2[] = {&add_c1, &x, &ms, &w, &y};
  return emmy_launch(apply, grid2, block2, 0, nullptr, p2, stream);
}

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
// (two streams, two threads) race on it.
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
    if (e != cudaSuccess || !p)
      return fail_msg(EMMY_ENODRIVER, "emmy_rmsnorm_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(e));
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
    int rows, void *stream) {
  if (!meansq || !apply || !grid1 || !block1 || !grid2 || !block2 || !mean_count || !add_c1 ||
      !x || !w || !y)
    return emmy_internal_fail(EMMY_EINVAL, "emmy_rmsnorm_noalloc: bad argument");
  if (rows <= 0 || rows > EMMY_NOALLOC_MAX_ROWS)
    return fail_msg(EMMY_EINVAL,
                    "emmy_rmsnorm_noalloc: %s %ld rows, the scratch array holds 1..%ld",
                    "cannot take", rows, static_cast<long>(EMMY_NOALLOC_MAX_ROWS));
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

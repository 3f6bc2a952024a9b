/*
 * emmy_b200.h -- C ABI of the B200 (sm_100a) runtime for Emmy Kernel IR kernels.
 *
 * The reference (emmy-hackathon-2026) turns a Kernel IR into PTX with
 * `python compile.py kernel.ir.json > out.ptx` and hands that PTX to a runner
 * that assembles it with ptxas and launches it under the problem's meta.json
 * (grid, block, dynamic shared memory, positional pointer arguments, outputs
 * zeroed first).  The runner is either the hosted HTTP service
 * (reference docs/API.md:12-53, client submit.py:80-161) or the local ctypes
 * driver-API script (reference tools/harness/gpu_run.py:46-103).  This
 * library is the native replacement for both: every entry point below names
 * the reference interface it replaces.
 *
 * Conventions
 *  - Every function returns 0 on success.  A positive value is a CUresult from
 *    the CUDA driver; a negative value is one of the EMMY_E* codes.  The text
 *    of the last failure on the calling thread is emmy_last_error().
 *  - Device memory is plain `uint64_t` device addresses (CUdeviceptr); streams
 *    are `void *` (a CUstream / cudaStream_t, NULL = the legacy stream).
 *  - No torch or CUDA headers are needed to call this ABI.
 *  - The library loads libcuda.so.1 lazily on the first call that needs a GPU,
 *    so it loads (and assembles PTX) on machines without one.
 */
#ifndef EMMY_B200_H
#define EMMY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define EMMY_API __attribute__((visibility("default")))
#else
#define EMMY_API
#endif

#define EMMY_ABI_VERSION 1

enum {
  EMMY_OK = 0,
  EMMY_EINVAL = -1,      /* bad argument (size, pointer, rank, ...)          */
  EMMY_ENODRIVER = -2,   /* libcuda.so.1 missing or a symbol not found       */
  EMMY_EPTXAS = -3,      /* PTX failed to assemble (log in emmy_last_error)  */
  EMMY_ENOENT = -4,      /* kernel entry or module global not found          */
  EMMY_EKERNEL = -5,     /* a kernel reported a failure through its error word */
  EMMY_ENOMEM = -6       /* host allocation failed                            */
};

/* Opaque handles. */
typedef struct emmy_image_s *emmy_image_t;   /* an assembled cubin            */
typedef struct emmy_module_s *emmy_module_t; /* a module loaded on a device   */
typedef struct emmy_kernel_s *emmy_kernel_t; /* one `.entry` of a module      */

/* Library version (EMMY_ABI_VERSION) and last error text of this thread. */
EMMY_API int emmy_abi_version(void);
EMMY_API const char *emmy_last_error(void);

/* ------------------------------------------------------------------------ */
/* Assemble: replaces the runner's `POST /compile` (ptxas on the PTX text,   */
/* returns a cubin id and the register count; reference docs/API.md:12-24).  */
/* ptxas runs in-process (nvPTXCompiler).  `arch` is e.g. "sm_100a"; `opts`  */
/* are extra ptxas flags ("-O3", "--maxrregcount=N", ...).                   */
/* ------------------------------------------------------------------------ */
EMMY_API int emmy_ptx_assemble(const char *ptx, size_t ptx_len, const char *arch,
                      const char *const *opts, int n_opts, emmy_image_t *out);
EMMY_API int emmy_image_data(emmy_image_t img, const void **data, size_t *len);
/* ptxas's info log (registers, spills, shared memory) for this image. */
EMMY_API const char *emmy_image_log(emmy_image_t img);
EMMY_API void emmy_image_free(emmy_image_t img);

/* ------------------------------------------------------------------------ */
/* Device and modules: replaces cuInit / cuCtxCreate / cuModuleLoadData /    */
/* cuModuleGetFunction in reference tools/harness/gpu_run.py:47-66.  The     */
/* device's primary context is retained and made current, so device memory   */
/* from any runtime-API user of that device (e.g. a framework allocator) is  */
/* valid in kernel launches.                                                 */
/* ------------------------------------------------------------------------ */
EMMY_API int emmy_device_count(int *count);
EMMY_API int emmy_device_init(int device);
EMMY_API int emmy_module_load(const void *image, size_t len, emmy_module_t *out);
EMMY_API int emmy_module_unload(emmy_module_t mod);
EMMY_API int emmy_kernel_get(emmy_module_t mod, const char *entry, emmy_kernel_t *out);
/* Registers per thread, static shared bytes, max threads per block. */
EMMY_API int emmy_kernel_attrs(emmy_kernel_t k, int *regs, int *static_smem, int *max_threads);
/* Address and size of a module-scope `.global` variable (e.g. the error word
 * `__emmy_status` that bounded waits in the kernels write). */
EMMY_API int emmy_module_global(emmy_module_t mod, const char *name, uint64_t *dptr, size_t *bytes);

/* ------------------------------------------------------------------------ */
/* Tensor maps: the reference IR declares TMA descriptors as "host-built"    */
/* (reference TASK.md:130, TmaDescriptor).  Encodes one tiled CUtensorMap    */
/* (128 bytes, written to `tmap`).  dtype: 0=u8 1=u16 2=u32 3=i32 4=u64       */
/* 5=i64 6=f16 7=f32 8=f64 9=bf16 10=tf32 (CUtensorMapDataType numbering).    */
/* dims/strides are innermost-first; strides[i] is the byte stride of        */
/* dimension i+1 (rank-1 values).  swizzle (CUtensorMapSwizzle numbering):  */
/* 0 none, 1 32B, 2 64B, 3 128B, 4 128B with 32B atoms, 5 the same with the */
/* 8-byte flip, 6 128B with 64B atoms.                                       */
/* ------------------------------------------------------------------------ */
EMMY_API int emmy_tensormap_encode(void *tmap, int dtype, int rank, uint64_t gaddr,
                          const uint64_t *dims, const uint64_t *strides,
                          const uint32_t *box, int swizzle);

/* ------------------------------------------------------------------------ */
/* Launch: replaces cuLaunchKernel under the meta.json geometry (reference   */
/* tools/harness/gpu_run.py:82-90; runner `POST /run`, docs/API.md:26-53).   */
/* `params[i]` points at the value of parameter i (cuLaunchKernel layout:    */
/* the meta arg_order pointers, then any host-built tensor maps the PTX      */
/* declares).  Dynamic shared memory above 48 KiB is opted in here, as the   */
/* reference runner does with cuFuncSetAttribute (gpu_run.py:87-88).         */
/* cluster[3] may be NULL (no cluster).                                      */
/* ------------------------------------------------------------------------ */
EMMY_API int emmy_launch(emmy_kernel_t k, const uint32_t grid[3], const uint32_t block[3],
                uint32_t smem_bytes, const uint32_t *cluster, void **params, void *stream);

/* `zero_outputs`: memset of output buffers before every launch
 * (reference docs/API.md:52-53). */
EMMY_API int emmy_memset_async(uint64_t dptr, int byte_value, size_t bytes, void *stream);
EMMY_API int emmy_memcpy_htod_async(uint64_t dst, const void *src, size_t bytes, void *stream);
EMMY_API int emmy_memcpy_dtoh_async(void *dst, uint64_t src, size_t bytes, void *stream);
EMMY_API int emmy_stream_sync(void *stream);

/* Device memory for callers that have no allocator of their own (the CPU-side
 * harness in tests); framework users pass their own device pointers instead. */
EMMY_API int emmy_mem_alloc(uint64_t *dptr, size_t bytes);
EMMY_API int emmy_mem_free(uint64_t dptr);

/* ------------------------------------------------------------------------ */
/* Peer memory between the processes of one multi-GPU job (one process per   */
/* GPU).  The reference is single-GPU and has no counterpart: these serve     */
/* the harness's cross-GPU finish of the global sum (the host side of         */
/* emmy_b200/peer.py), which writes each rank's partial straight into every   */
/* peer's memory over NVLink.  `emmy_ipc_handle` exports an allocation made   */
/* by `emmy_mem_alloc` (64 opaque bytes, exchanged by the caller);            */
/* `emmy_ipc_open` maps a peer's allocation into this process (peer access    */
/* enabled as needed) and `emmy_ipc_close` unmaps it.                        */
/* ------------------------------------------------------------------------ */
EMMY_API int emmy_ipc_handle(uint64_t dptr, unsigned char handle_out[64]);
EMMY_API int emmy_ipc_open(const unsigned char handle[64], uint64_t *dptr_out);
EMMY_API int emmy_ipc_close(uint64_t dptr);

/* ------------------------------------------------------------------------ */
/* Timing: the runner reports `median_us` over `iters` launches after         */
/* `warmup` (reference docs/API.md:15-36).  This launches `iters` times       */
/* back to back on `stream`, records a CUDA event pair around each launch,    */
/* and between launches (outside the events) optionally writes `flush_bytes`  */
/* of `flush_dptr` to evict L2, then drops that buffer's lines from L2 with   */
/* discard.global.L2 (so no dirty line of the flush is written back inside a  */
/* timed launch), and re-zeroes `n_zero` output buffers.                      */
/* ms_out receives `iters` per-launch times in milliseconds.                  */
/* ------------------------------------------------------------------------ */
EMMY_API int emmy_time_launches(emmy_kernel_t k, const uint32_t grid[3], const uint32_t block[3],
                       uint32_t smem_bytes, const uint32_t *cluster, void **params,
                       void *stream, int warmup, int iters,
                       uint64_t flush_dptr, size_t flush_bytes,
                       const uint64_t *zero_dptrs, const size_t *zero_bytes, int n_zero,
                       float *ms_out);

/* ------------------------------------------------------------------------ */
/* Host-buffer run: the whole `POST /run` round trip for a caller holding    */
/* host memory (reference docs/API.md:26-53 "args", submit.py:126-135):       */
/* copy every input to its device buffer, zero the outputs, launch, copy the  */
/* outputs back.  n_args buffers in arg_order; is_output[i] selects direction.*/
/* dev[i] are caller-owned device buffers of bytes[i] bytes.  An input with  */
/* bytes[i] == 0 is not copied: its device buffer already holds the data     */
/* (e.g. copied by an earlier call of the same step for another kernel).     */
/* ------------------------------------------------------------------------ */
EMMY_API int emmy_run_host(emmy_kernel_t k, const uint32_t grid[3], const uint32_t block[3],
                  uint32_t smem_bytes, const uint32_t *cluster, int n_args,
                  void *const *host, const uint64_t *dev, const size_t *bytes,
                  const int *is_output, int n_extra, void **extra_params, void *stream);

/* ------------------------------------------------------------------------ */
/* No counterpart in the reference (its runner allocates every buffer).      */
/* For callers that cannot allocate device memory when they call in -- an    */
/* allocator that owns all device memory, code running while a CUDA graph   */
/* is built, a fixed memory budget: the two-kernel RMSNorm (`meansq` = row   */
/* mean of squares into an intermediate, then `apply` = x * rsqrt(ms + eps)  */
/* * w; the pair compiled from those two IRs for exactly rows x cols, params */
/* in their meta arg_order) with the intermediate in a static device array  */
/* of EMMY_NOALLOC_MAX_ROWS floats (256 KiB, held by every GPU that loads    */
/* the library until exit) instead of a caller buffer.  The caller passes    */
/* inputs (the one-element constant buffers mean_count and add_c1,          */
/* x[rows, cols], w[cols]) and the output y.  Refused with EMMY_EINVAL      */
/* before anything runs: more rows than the array holds, a grid1 other than */
/* (rows, 1, 1) (the first kernel writes one entry per CTA), or a 1-D       */
/* grid2 x block2 that does not cover rows x cols elements with less than   */
/* one block to spare (the second reads one entry per element's row).      */
/* The first call on a device loads the library's device code there and    */
/* so reserves the array on that device: make it at start-up if the memory */
/* budget is fixed, and before any stream capture.  All calls share the     */
/* array, so calls that overlap on the GPU race.  The calls themselves      */
/* allocate nothing.                                                         */
/* ------------------------------------------------------------------------ */
#define EMMY_NOALLOC_MAX_ROWS 65536
EMMY_API int emmy_rmsnorm_noalloc(emmy_kernel_t meansq, const uint32_t grid1[3],
                                  const uint32_t block1[3], emmy_kernel_t apply,
                                  const uint32_t grid2[3], const uint32_t block2[3],
                                  uint64_t mean_count, uint64_t add_c1, uint64_t x, uint64_t w,
                                  uint64_t y, int rows, int cols, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* EMMY_B200_H */

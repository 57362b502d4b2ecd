/*
 * commux_strided_copy_noalloc: a strided device-to-device copy on one GPU that
 * allocates nothing.
 *
 * No counterpart in the reference: the reference's UCX backend stages device
 * data through `.contiguous()` copies and UCX's own buffers. This entry point
 * exists for callers that must not allocate device memory at the time of the
 * copy:
 *
 *   - code that runs while the PyTorch caching allocator cannot be entered,
 *     such as an out-of-memory handler or an allocator callback: asking the
 *     allocator for scratch there re-enters it;
 *   - serving processes that reserve their whole device-memory budget at start
 *     and treat any later allocation as a failure;
 *   - latency-critical loops: cudaMalloc and cudaFree may synchronise the
 *     whole device, stalling every other stream;
 *   - plain C or C++ programs that own their buffers and have no PyTorch
 *     allocator to borrow scratch from.
 *
 * The copy runs the same pull kernel that moves tagged p2p messages (a
 * strided gather from `src` and a strided scatter into `dst` in one pass,
 * vectorised up to 16 bytes). The only scratch the kernel needs, its
 * per-descriptor completion counters and flags, lives in a file-scope device
 * array of 1 KiB per GPU that is compiled into the library, so the call performs no
 * cudaMalloc, cudaFree or other allocating CUDA or PyTorch routine, and no
 * host heap allocation either.
 *
 * Semantics:
 *   - copies the `ndim`-dimensional view (`sizes`, `src_strides`) at `src`
 *     into the view (`sizes`, `dst_strides`) at `dst`; strides are in
 *     elements of `elem_bytes` bytes (1, 2, 4, 8 or 16); ndim <= 8;
 *   - both views must lie inside one device allocation each, on the current
 *     device, and must not overlap; the call checks the first, not the second;
 *   - asynchronous on `stream` (a cudaStream_t, NULL = the legacy default
 *     stream), which must belong to the current device;
 *   - before its copy kernel, each call clears the counters and flags on
 *     `stream` with a small kernel of its own (they must start at zero).
 *
 * Limits (oversize inputs are rejected with CMX_NOALLOC_ETOOBIG and a message,
 * before any memory is touched):
 *   - at most 64 copy descriptors per call: a descriptor covers at most 2^30
 *     vector units (1 TiB in total at 16-byte units), split along the
 *     outermost dimension;
 *   - the dimensions inside the outermost one together hold at most 2^30
 *     units;
 *   - at most 4 dimensions remain after dropping size-1 dimensions and merging
 *     those contiguous in both views (else CMX_NOALLOC_ELAYOUT).
 *
 * Concurrency: every call on a device shares that device's one scratch array.
 * Calls whose kernels may overlap (other streams, other host threads without
 * ordering between them) race on the counters and can produce a wrong copy;
 * issue them on one stream or order them with events.
 *
 * Set-up: the first call on each device looks up the scratch array's device
 * address (cudaGetSymbolAddress) and loads every kernel a later call can
 * launch (by default CUDA loads a kernel lazily at its first launch, and a
 * load may allocate device memory). That first call may therefore allocate;
 * no later call does. Make the first call on each device before any stream
 * capture begins, and outside the code that must not allocate.
 *
 * Context: the call runs in the device's primary context, the one the CUDA
 * runtime uses; it does not change the calling thread's current device or
 * context. A thread that made another driver context current gets
 * CMX_NOALLOC_EINVAL until it makes the primary context current again. The
 * cached set-up belongs to the primary context: after a cudaDeviceReset the
 * next call repeats the set-up when the new primary context has a new handle,
 * but a handle can be reused, so do not mix this call with cudaDeviceReset.
 *
 * Returns CMX_NOALLOC_OK (0) or an error code; on error a NUL-terminated
 * message is written to `err` (at most `err_len` bytes, may be NULL).
 */
#ifndef COMMUX_NOALLOC_H_
#define COMMUX_NOALLOC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  CMX_NOALLOC_OK = 0,
  CMX_NOALLOC_EINVAL = 1,   /* bad argument (pointer, ndim, elem_bytes, alignment), or a
                               context other than the device's primary one is current */
  CMX_NOALLOC_ETOOBIG = 2,  /* more descriptors or units than the static scratch covers */
  CMX_NOALLOC_ELAYOUT = 3,  /* more than 4 dims after merging */
  CMX_NOALLOC_ERANGE = 4,   /* a view leaves its allocation or is not on the current device */
  CMX_NOALLOC_ECUDA = 5     /* a CUDA call failed (set-up, memset or launch) */
};

int commux_strided_copy_noalloc(void* dst, const int64_t* dst_strides, const void* src,
                                const int64_t* src_strides, const int64_t* sizes, int ndim,
                                int elem_bytes, void* stream, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* COMMUX_NOALLOC_H_ */

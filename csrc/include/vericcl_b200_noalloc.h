/* vericcl_b200: a single-GPU AllReduce entry point that allocates no memory.
 *
 * This entry point has no counterpart in the reference implementation.
 *
 * Who it is for: callers that must not allocate device memory on their call
 * path - a plug-in running inside a host application that owns every byte of
 * device memory, code that runs under a fixed device-memory budget where a
 * new allocation may fail or stall, and C/C++ callers that link no CUDA
 * allocator at all (no PyTorch, no caching allocator) and cannot hand this
 * library a symmetric heap.  The regular paths (the PyTorch extension and
 * vb_execute) stage data through heap buffers created with cudaMalloc /
 * cuMemCreate; this one uses a fixed static device array instead.
 *
 * What it does: out = scale * in for `count` elements on one GPU - the
 * single-rank AllReduce of a synthesized schedule with its fused scale, run by
 * the same schedule-interpreter kernel as every other collective.  The
 * interpreter's working memory - its control block, its flag table, its
 * compiled one-step program and the staging buffer the schedule runs on - lives
 * in one file-scope `static __device__ __align__(256)` array of
 * VB_NOALLOC_SCRATCH_BYTES (8 MiB).  Every GPU that loads the library holds
 * that array until the process exits.  The call copies `in` into the staging
 * buffer, launches the interpreter, and copies the result to `out`, all
 * enqueued on `cuda_stream`; it calls no cudaMalloc, cudaFree or any other
 * allocating routine.
 *
 * Limits and rules:
 *  - count * element size must not exceed VB_NOALLOC_MAX_BYTES; larger
 *    requests are rejected with VB_NOALLOC_TOO_LARGE before anything is
 *    enqueued (vb_noalloc_last_error() explains why).
 *  - The first call on a device performs the set-up for that device: with the
 *    device current it looks up the array's device address
 *    (cudaGetSymbolAddress), clears the control block and flag table, and
 *    writes the program.  Make that first call before any stream capture.
 *  - Every call on a device shares the same array, which keeps the last call's
 *    contents between calls (each call clears the status words that must
 *    start at zero).  Calls whose GPU work overlaps - for example on two
 *    streams at once - race on the array; serialise them on one stream.
 *  - The kernel never hangs: its waits are bounded and a failure is written
 *    to a status word in the array instead of trapping.  After synchronising
 *    the stream, vb_noalloc_status() reports it; on a failure `out` holds
 *    the unscaled input and must not be used.
 *  - The set-up belongs to the device's current CUDA context.  A call made
 *    under a different context (after cudaDeviceReset, for example) repeats
 *    the set-up for that context.
 */
#ifndef VERICCL_B200_NOALLOC_H
#define VERICCL_B200_NOALLOC_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VB_NOALLOC_SCRATCH_BYTES (8u << 20)
#define VB_NOALLOC_RESERVED_BYTES (64u << 10)
#define VB_NOALLOC_MAX_BYTES (VB_NOALLOC_SCRATCH_BYTES - VB_NOALLOC_RESERVED_BYTES)

enum {
  VB_NOALLOC_OK = 0,
  VB_NOALLOC_INVALID = 1,    /* null pointer, zero count, unknown dtype */
  VB_NOALLOC_TOO_LARGE = 2,  /* count * element size exceeds VB_NOALLOC_MAX_BYTES */
  VB_NOALLOC_CUDA_ERROR = 3  /* a CUDA call failed (symbol lookup, copy, launch) */
};

/* dtype: 0 float32, 1 bfloat16, 2 float16.  in/out are device pointers (may be equal). */
int vb_allreduce_local_noalloc(const void* in, void* out, size_t count, int dtype, float scale, void* cuda_stream);

/* The kernel status of the last call on the current device: *status is 0 when
 * it completed, 1 when a wait ran out of time, 2 when it was aborted, 3 for a
 * bad geometry; detail (may be NULL) receives rank, block, lane and wait index
 * of the failure.  Synchronise the call's stream first.  Returns VB_NOALLOC_OK
 * or VB_NOALLOC_CUDA_ERROR. */
int vb_noalloc_status(int* status, int detail[4]);

/* Human-readable reason of the calling thread's last failed call. */
const char* vb_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif

#endif

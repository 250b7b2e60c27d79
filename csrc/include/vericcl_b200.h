/* vericcl_b200 C API: execute a synthesized collective schedule from C/C++.
 *
 * One context per rank (one process per GPU).  All calls except
 * vb_status/vb_last_error are collective: every rank makes the same calls in
 * the same order.  Every call has a deadline; a call whose GPU work does not
 * finish in time returns VB_UNRESOLVED, raises the device abort word so the
 * interpreter's bounded waits end early, and keeps ownership of its buffers
 * (vb_close never frees memory that is still in use).
 */
#ifndef VERICCL_B200_H
#define VERICCL_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VERICCL_B200_ABI_VERSION 2

typedef enum vb_result {
  VB_OK = 0,
  VB_INVALID = 1,     /* bad argument or schedule */
  VB_BUSY = 2,        /* another call is active on this context */
  VB_TIMEOUT = 3,     /* a control phase did not complete before its deadline */
  VB_UNRESOLVED = 4,  /* GPU work did not finish before its deadline; buffers stay owned */
  VB_FAILED = 5,      /* CUDA or device failure */
  VB_CLOSED = 6       /* the context was closed */
} vb_result;

typedef enum vb_dtype { VB_FLOAT32 = 0, VB_BFLOAT16 = 1, VB_FLOAT16 = 2 } vb_dtype;
typedef enum vb_redop { VB_SUM = 0, VB_PROD = 1, VB_MIN = 2, VB_MAX = 3 } vb_redop;

typedef struct vb_init_params {
  int abi_version;            /* VERICCL_B200_ABI_VERSION */
  int rank, nranks, device;
  const char* control_address;   /* IPv4 address of rank 0's coordinator */
  int control_port;
  const char* session;        /* identical on every rank */
  double timeout_s;           /* deadline of this call */
  size_t heap_bytes;          /* symmetric heap per rank */
  int multicast;              /* bind the heap to an NVLS multicast object when possible */
} vb_init_params;

typedef struct vb_context vb_context;

vb_result vb_init(const vb_init_params* params, vb_context** out);
/* Compile the XML schedule for this rank and agree on its sha256 with every rank. */
vb_result vb_prepare(vb_context* ctx, const char* xml, int nlanes, int niters, double timeout_s);
/* Run the prepared schedule: count input elements per rank from `in` to `out` (device pointers). */
vb_result vb_execute(vb_context* ctx, const void* in, void* out, size_t count, int dtype, int redop, float scale,
                     void* cuda_stream, double timeout_s);
/* Device status word (0 ok, 1 timeout, 2 aborted, 3 bad geometry) and launch epoch; never blocks. */
vb_result vb_status(vb_context* ctx, int* device_status, unsigned long long* epoch);
/* Record per-step timestamps in the next vb_execute (after vb_prepare; not collective). */
vb_result vb_trace_arm(vb_context* ctx);
/* Write the traced execution of this rank as a trace file (40-byte header, 64-byte records). */
vb_result vb_trace_write(vb_context* ctx, const char* path);
vb_result vb_release(vb_context* ctx);
vb_result vb_close(vb_context* ctx, double timeout_s);
vb_result vb_destroy(vb_context* ctx);
const char* vb_last_error(vb_context* ctx);
int vb_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif

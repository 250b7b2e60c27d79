// Kernel launch arguments and launch entry points of the schedule interpreter.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "vb/devprog.h"

namespace vb {

// Status words written by the kernels (local device memory).
enum StatusCode : int {
  ST_OK = 0,
  ST_TIMEOUT = 1,        // a flag wait exceeded its time limit
  ST_ABORTED = 2,        // another CTA or the host requested an abort
  ST_BAD_GEOMETRY = 3,   // a piece or address was out of range / misaligned
};

struct Control {
  unsigned long long epoch;       // launch counter of this communicator (starts at 1)
  unsigned int arrive;            // CTAs finished in the current launch
  int status;                     // StatusCode of the first failure
  int detail[4];                  // rank, block, lane, wait index of the first failure
  int abort_request;              // host-set abort flag (mapped memory or device write)
  unsigned int ll_arrive;         // CTAs finished in the current one-shot launch
  unsigned long long ll_seq;      // one-shot launch counter (tags the flag-in-data lines)
  unsigned long long fp8_seq;     // fused fp8 AllGather launch counter (its staging parity and flag values)
  unsigned int fp8_arrive;        // CTAs finished in the current fused fp8 AllGather launch
  unsigned int push_arrive;       // CTAs finished in the current push AllGather launch
  unsigned long long push_seq;    // push AllGather launch counter (its start and done flag values)
  unsigned long long pace_clock;  // link emulation: %globaltimer until which this rank's emulated link is busy
};
static_assert(sizeof(Control) <= 256, "workspaces reserve 256 bytes for the control block");

struct InterpArgs {
  const DevBlock* blocks;
  const DevStep* steps;
  const DevSrc* srcs;
  const DevWait* waits;
  int nblocks, nlanes, niters, rank, nranks;
  int dtype, redop;
  float scale;
  long long chunk_elems, piece_elems;
  long long buf_off[BUF_COUNT];      // byte offsets inside the heap (identical on all ranks)
  long long batch_stride[BUF_COUNT]; // byte distance between consecutive batched instances of a buffer
  int nbatch;                        // instances of the program run back to back in this launch
  long long flag_off;                // byte offset of the flag table inside the heap
  long long start_slot;              // flag index of the per-rank start flag
  char* base[kMaxRanks];             // heap base of every rank in this process's address space
  char* mc_base;                     // multicast address of the heap (nullptr when unavailable)
  Control* control;                  // local control block
  unsigned long long timeout_ns;
  int pace_group;                    // >0: emulate slow links between rank groups of this size
  float pace_ns_per_byte;            // emulated link time per byte this rank reads from another group
  int trace;                         // record per-step timestamps into trace buffer
  unsigned long long* trace_buf;     // [nblocks*nlanes][max_steps*niters][2] (start, end) globaltimer
  int trace_stride;
  // Optional launch timeline: [kTimelineSlots][2] %globaltimer of kernel entry (CTA 0) and exit (last CTA to
  // finish), indexed by launch epoch modulo kTimelineSlots; nullptr disables it (separate kernel instance).
  unsigned long long* timeline;
  int lean;                          // 1: run the register-lean kernel instance (sum reductions and copies)
  int bulk;                          // bit 0: copy and reduce steps stage their sources in shared memory with TMA
                                     //    bulk copies (cp.async.bulk) instead of per-thread vector loads;
                                     // bit 1: staged plain copies into local memory are also written back by TMA
};

// TMA staging of copy/reduce sources: kBulkStages buffers of kBulkStageBytes each, one mbarrier per buffer.
constexpr int kBulkStages = 3;
constexpr int kBulkStageBytes = 64 * 1024;
constexpr int kBulkSmemBytes = kBulkStages * kBulkStageBytes + 128;
constexpr long long kBulkMinBytes = 32 * 1024;   // smaller pieces keep the per-thread vector path

constexpr int kTimelineSlots = 256;

// Launch the interpreter (cooperative launch: every CTA is co-resident).
cudaError_t launch_interp(const InterpArgs& args, cudaStream_t stream, int threads);
int interp_max_ctas(int threads);
// Inter-group link emulation from VERICCL_EMULATE (off when unset).
void apply_emulation_env(InterpArgs* a);

// Helper kernels.
cudaError_t launch_fill(void* dst, long long n, int dtype, int pattern, int rank, unsigned long long seed,
                        cudaStream_t stream);
cudaError_t launch_scale(void* dst, const void* src, long long n, int dtype, float scale, cudaStream_t stream);
cudaError_t launch_strided_copy(void* dst, long long dst_pitch, const void* src, long long src_pitch,
                                long long row_bytes, long long rows, cudaStream_t stream);
// Counts outputs that differ from the analytic result of pattern-0 inputs.  collective: 0 allreduce,
// 1 allgather, 2 reduce_scatter, 3 broadcast, 4 reduce (root), 5 alltoall, 6 the rank's own input.
cudaError_t launch_check(const void* out, long long n, int dtype, int collective, int redop, int nranks,
                         int rank, long long count_per_rank, double atol, double rtol, unsigned long long* bad,
                         cudaStream_t stream, int root = 0, double scale = 1.0);
cudaError_t launch_read_timer(unsigned long long* dst, cudaStream_t stream);

// Block-scaled FP8 (e4m3) payloads.
cudaError_t launch_quantize_fp8(const void* in, unsigned char* q, float* scales, long long n, int block, int dtype,
                                cudaStream_t stream);
cudaError_t launch_dequantize_fp8(const unsigned char* q, const float* scales, void* out, long long n, int block,
                                  int dtype, cudaStream_t stream);

// One-shot low-latency AllReduce / AllGather (flag-in-data lines pushed into every peer's LL region).
enum OneShotColl : int { OS_ALLREDUCE = 0, OS_ALLGATHER = 1, OS_ALLREDUCE_TWOSHOT = 2 };

struct OneShotArgs {
  char* base[kMaxRanks];     // heap base of every rank in this process's address space
  long long in_off, out_off; // byte offsets of this call's buffers (identical on all ranks)
  long long ll_off;          // byte offset of the LL region: [2 parities][nranks sources][bytes/8 lines of 16 B]
  long long ll_src_bytes;    // bytes of one source's lines (>= 2 * bytes)
  long long bytes;           // payload bytes per rank (multiple of 8)
  int rank, nranks, dtype, redop, coll;
  float scale;
  int do_scale;
  Control* control;
  unsigned long long timeout_ns;
  char* mc_base;             // multicast address of the heap: one NVLS store reaches every rank (nullptr: unicast)
};

// Bytes of LL region needed for payloads up to max_bytes per rank.
long long oneshot_region_bytes(int nranks, long long max_bytes);
cudaError_t launch_oneshot(const OneShotArgs& args, cudaStream_t stream);
int oneshot_max_ctas();

// Fused block-scaled FP8 AllGather: one launch quantizes this rank's input into its staging area
// (e4m3 bytes + one fp32 scale per 128 elements), publishes per-CTA flags, pulls every peer's staging
// over NVLink and dequantizes it straight into the output.  Staging and flags live in the symmetric
// heap at the same offsets on every rank; the staging area holds two parities of fp8_stage_bytes(n).
struct Fp8AgArgs {
  char* base[kMaxRanks];     // heap base of every rank in this process's address space
  const void* in;            // this rank's n input elements (any device memory)
  void* out;                 // nranks * n output elements (any device memory)
  long long n;               // elements per rank (multiple of 16)
  long long stage_off;       // heap offset of the two staging parities
  long long flag_off;        // heap offset of the per-CTA flags ([ctas] u64 per rank)
  int rank, nranks, dtype, ctas;
  Control* control;
  unsigned long long timeout_ns;
};
long long fp8_stage_bytes(long long n);        // bytes of one staging parity for n elements
cudaError_t launch_fp8_allgather(const Fp8AgArgs& args, cudaStream_t stream);
int fp8_allgather_max_ctas();

// Push AllGather: every rank stores its chunk straight into every peer's output (NVLink writes, no read
// requests travelling against the data), after the peer has entered the same launch; per-CTA done flags tell
// each receiver when the matching range of every part has landed.
struct PushAgArgs {
  char* base[kMaxRanks];     // heap base of every rank in this process's address space
  const void* in;            // this rank's chunk (local device memory)
  long long out_off;         // heap offset of the output (nranks * bytes), identical on every rank
  long long bytes;           // bytes per rank (multiple of 16)
  long long flag_off;        // heap offset of the flags: [0] start flag, [1 + c] done flag of CTA c
  int rank, nranks, ctas;
  int fanout;                // 0: one peer after another (re-reading the chunk); 1: each loaded vector to every rank
  Control* control;
  unsigned long long timeout_ns;
};
cudaError_t launch_push_allgather(const PushAgArgs& args, cudaStream_t stream);
int push_allgather_max_ctas();

// Calibration probes.
cudaError_t launch_copy_probe(void* dst, const void* src, long long bytes, int ctas, int threads, int unroll,
                              cudaStream_t stream);
cudaError_t launch_reduce_probe(void* dst, const void* const* srcs, int k, long long bytes, int ctas, int threads,
                                cudaStream_t stream);

}  // namespace vb

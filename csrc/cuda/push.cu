// Push AllGather for sm_100a: NVLink writes instead of reads.
//
// A pull moves data against a stream of read requests on the same links; when
// every GPU both sends and receives (an AllGather), the requests of one
// direction share the links with the data of the other, and a pull measured
// about 667 GB/s per direction with both GPUs of a pair pulling at once
// against about 770 GB/s alone.  Here every rank stores its own chunk into
// every peer's output instead, so only data (and small write acknowledgements)
// crosses the switch.
//
// Protocol of launch `seq` (a per-rank counter in the control block that every
// rank advances identically, one step per launch):
//  1. CTA 0 publishes the rank's start flag = seq + 1: from now on peers may
//     write into this rank's output (the output's previous contents belong to
//     work the stream has already finished).
//  2. CTA c owns bytes [c·B/C, (c+1)·B/C) of the chunk (16-byte units): it
//     copies them into its own output part, then for every peer q (rank + 1,
//     rank + 2, ...) waits until q's start flag reaches seq + 1 and stores them
//     into part `rank` of q's output.  In fan-out mode the CTA first waits for
//     every peer's start flag, then reads each vector of its range once and
//     stores it into every rank's output (own first, then rank + 1, ...): one
//     HBM read per byte instead of one per peer, and all of the GPU's links
//     busy from the first vector on.
//  3. Each thread fences its stores at system scope; after a CTA barrier,
//     thread 0 publishes this CTA's done flag = seq + 1 with st.release.sys.
//  4. CTA c then waits until the done flag of CTA c on every peer reaches
//     seq + 1: the c-th range of every part of this rank's output has landed.
// A rank's launch therefore ends only after every push into it has completed,
// and a rank pushes into a peer only after the peer entered the same launch,
// so launches may reuse the same buffers back to back.  Every wait is bounded
// by %globaltimer; on expiry the failure goes to the control block's status
// word (which stops the other waiters) and the CTA returns.
#include <cuda_runtime.h>

#include <cstdint>

#include "vb/launch.h"

namespace vb {
namespace {

constexpr int kPushThreads = 512;
constexpr int kPushUnroll = 4;

__device__ __forceinline__ unsigned long long push_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long push_ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void push_st_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint4 push_ld(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void push_st(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// dst[v] = src[v] for 16-byte vectors v in [0, nvec), kPushUnroll loads in flight per thread
__device__ __forceinline__ void copy_range(char* dst, const char* src, long long nvec) {
  const long long stride = (long long)kPushThreads * kPushUnroll;
  for (long long v0 = threadIdx.x; v0 < nvec; v0 += stride) {
    uint4 r[kPushUnroll];
#pragma unroll
    for (int u = 0; u < kPushUnroll; ++u) {
      const long long v = v0 + (long long)u * kPushThreads;
      if (v < nvec) r[u] = push_ld(src + v * 16);
    }
#pragma unroll
    for (int u = 0; u < kPushUnroll; ++u) {
      const long long v = v0 + (long long)u * kPushThreads;
      if (v < nvec) push_st(dst + v * 16, r[u]);
    }
  }
}

// Fan-out: each vector of [0, nvec) read once and stored into part `rank` of every rank's output.
__device__ __forceinline__ void fanout_range(const PushAgArgs& a, long long part, const char* src, long long nvec) {
  const long long stride = (long long)kPushThreads * kPushUnroll;
  for (long long v0 = threadIdx.x; v0 < nvec; v0 += stride) {
    uint4 r[kPushUnroll];
#pragma unroll
    for (int u = 0; u < kPushUnroll; ++u) {
      const long long v = v0 + (long long)u * kPushThreads;
      if (v < nvec) r[u] = push_ld(src + v * 16);
    }
    for (int step = 0; step < a.nranks; ++step) {
      const int q = a.rank + step < a.nranks ? a.rank + step : a.rank + step - a.nranks;
      char* dst = a.base[q] + a.out_off + part;
#pragma unroll
      for (int u = 0; u < kPushUnroll; ++u) {
        const long long v = v0 + (long long)u * kPushThreads;
        if (v < nvec) push_st(dst + v * 16, r[u]);
      }
    }
  }
}

__device__ void push_fail(const PushAgArgs& a, int peer, int what) {
  if (atomicCAS(&a.control->status, ST_OK, ST_TIMEOUT) == ST_OK) {
    a.control->detail[0] = a.rank;
    a.control->detail[1] = peer;
    a.control->detail[2] = blockIdx.x;
    a.control->detail[3] = what;
  }
  __threadfence();
}

// Thread 0 waits until *f >= target; returns false (and has recorded why) when the CTA must stop.
__device__ bool push_wait(const PushAgArgs& a, const unsigned long long* f, unsigned long long target, int peer,
                          int what) {
  if (push_ld_acquire(f) >= target) return true;
  const unsigned long long t0 = push_timer();
  unsigned int spins = 0;
  while (push_ld_acquire(f) < target) {
    if ((++spins & 63u) == 0) {
      if (*(volatile int*)&a.control->status != ST_OK || *(volatile int*)&a.control->abort_request) return false;
      if (push_timer() - t0 > a.timeout_ns) {
        push_fail(a, peer, what);
        return false;
      }
    }
  }
  return true;
}

__global__ void __launch_bounds__(kPushThreads, 1) push_allgather_kernel(const PushAgArgs a) {
  __shared__ unsigned long long s_seq;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_seq = *(volatile unsigned long long*)&a.control->push_seq;
    s_ok = 1;
  }
  __syncthreads();
  const unsigned long long seq = s_seq;
  unsigned long long* my_flags = reinterpret_cast<unsigned long long*>(a.base[a.rank] + a.flag_off);
  if (blockIdx.x == 0 && threadIdx.x == 0) push_st_release(my_flags, seq + 1);
  const long long nvec = a.bytes / 16;
  const long long v0 = nvec * blockIdx.x / a.ctas, v1 = nvec * (blockIdx.x + 1) / a.ctas;
  const char* src = static_cast<const char*>(a.in) + v0 * 16;
  const long long part = (long long)a.rank * a.bytes + v0 * 16;
  if (a.fanout) {
    if (threadIdx.x == 0) {
      for (int step = 1; step < a.nranks; ++step) {
        const int q = (a.rank + step) % a.nranks;
        const unsigned long long* start = reinterpret_cast<const unsigned long long*>(a.base[q] + a.flag_off);
        if (!push_wait(a, start, seq + 1, q, 0)) {
          s_ok = 0;
          break;
        }
      }
    }
    __syncthreads();
    if (s_ok) fanout_range(a, part, src, v1 - v0);
  } else {
    copy_range(a.base[a.rank] + a.out_off + part, src, v1 - v0);
    for (int step = 1; step < a.nranks; ++step) {
      const int q = (a.rank + step) % a.nranks;
      if (threadIdx.x == 0) {
        const unsigned long long* start = reinterpret_cast<const unsigned long long*>(a.base[q] + a.flag_off);
        if (!push_wait(a, start, seq + 1, q, 0)) s_ok = 0;
      }
      __syncthreads();
      if (!s_ok) break;
      copy_range(a.base[q] + a.out_off + part, src, v1 - v0);
    }
  }
  // every thread's remote stores reach their targets before this CTA's done flag does
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0 && s_ok) push_st_release(my_flags + 1 + blockIdx.x, seq + 1);
  if (threadIdx.x == 0 && s_ok) {
    for (int step = 1; step < a.nranks; ++step) {
      const int q = (a.rank + step) % a.nranks;
      const unsigned long long* done = reinterpret_cast<const unsigned long long*>(a.base[q] + a.flag_off) + 1 +
                                       blockIdx.x;
      if (!push_wait(a, done, seq + 1, q, 1)) break;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.control->push_arrive, 1u) == gridDim.x - 1) {
      a.control->push_arrive = 0;
      a.control->push_seq = seq + 1;
      __threadfence();
    }
  }
}

}  // namespace

int push_allgather_max_ctas() {
  static int cached[64] = {};
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, push_allgather_kernel, kPushThreads, 0);
  const int v = sms * per_sm;
  if (dev >= 0 && dev < 64) cached[dev] = v;
  return v;
}

cudaError_t launch_push_allgather(const PushAgArgs& a, cudaStream_t stream) {
  if (a.bytes <= 0 || a.bytes % 16 || a.ctas < 1 || a.nranks < 1 || a.nranks > kMaxRanks || a.rank < 0 ||
      a.rank >= a.nranks || a.ctas > push_allgather_max_ctas() || a.ctas > 4096)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.in) % 16 || a.out_off % 16 || a.flag_off % 8) return cudaErrorMisalignedAddress;
  void* args[] = {const_cast<PushAgArgs*>(&a)};
  // co-residency: CTA c on one rank waits for CTA c of every peer
  return cudaLaunchCooperativeKernel((void*)push_allgather_kernel, dim3(a.ctas), dim3(kPushThreads), args, 0, stream);
}

}  // namespace vb

// One-shot low-latency AllReduce / AllGather for small messages on sm_100a.
//
// The interpreter's pull protocol costs two cross-GPU round trips per
// collective (arrival flags before the loads, completion waits before the
// kernel ends).  For messages of a few KiB to a few hundred KiB that latency
// dominates, so this path uses a flag-in-data protocol instead: every rank
// pushes its payload into a slot of every peer's LL region (with NVLS, one
// multicast store per 8-byte half reaches all of them), 8 payload bytes
// per 16-byte line {data0, tag, data1, tag} written as two 8-byte halves that
// are each single-copy atomic, and then reads the lines the peers pushed into
// its own region, waiting only until both tags of a line match this launch.
// No separate flag, fence or barrier is needed, and nothing ever reads a
// peer's buffers.
//
// Tags and slot reuse: the launch counter `ll_seq` lives in the rank's
// control block and advances once per launch (the last CTA to finish bumps
// it), identically on every rank because every rank runs the same sequence
// of collectives.  Lines of launch `seq` go to region half `seq & 1` with tag
// `seq mod (2^32 - 2) + 1`; the half still holds the tags of launch `seq - 2`,
// which never equal the current ones, and the region starts zeroed, which is
// no tag.  A half is rewritten two launches later, and a rank can reach launch
// `seq + 2` only after it has read every peer's lines of `seq + 1`, which each
// peer pushes after its own launch `seq` has finished reading, so a line is
// never overwritten before it has been consumed.
//
// AllReduce combines the ranks' contributions in rank order on every rank
// (bitwise-identical results everywhere), in fp32, with the fused scale.
// Every wait is bounded by %globaltimer: on expiry the thread records the
// failure in the control block (which stops every other waiting thread) and stops.
// Protocol family: NCCL's LL (8-byte data/flag pairs); this implementation,
// its region layout and its tag rule are this project's own.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "vb/launch.h"

namespace vb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_volatile_int(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 ld_payload(const char* p) {
  uint2 v;
  asm volatile("ld.global.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ void st_payload(char* p, uint2 v) {
  asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

// One LL line: two 8-byte elements {data | tag << 32}; each element access is single-copy atomic.
__device__ __forceinline__ void st_line(char* p, uint2 d, unsigned int tag) {
  const unsigned long long lo = (unsigned long long)d.x | ((unsigned long long)tag << 32);
  const unsigned long long hi = (unsigned long long)d.y | ((unsigned long long)tag << 32);
  asm volatile("st.volatile.global.v2.u64 [%0], {%1,%2};" ::"l"(p), "l"(lo), "l"(hi) : "memory");
}

// The same line through the multicast address: NVSwitch replicates it into every rank's region.
__device__ __forceinline__ void mc_st_line(char* p, uint2 d, unsigned int tag) {
  const unsigned long long lo = (unsigned long long)d.x | ((unsigned long long)tag << 32);
  const unsigned long long hi = (unsigned long long)d.y | ((unsigned long long)tag << 32);
  asm volatile("multimem.st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(lo) : "memory");
  asm volatile("multimem.st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p + 8), "l"(hi) : "memory");
}

__device__ __forceinline__ void ld_line(const char* p, unsigned long long& lo, unsigned long long& hi) {
  asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(lo), "=l"(hi) : "l"(p) : "memory");
}

// 8 payload bytes as floats.
template <int DT>
struct Unit;

template <>
struct Unit<DT_F32> {
  static constexpr int N = 2;
  __device__ static void unpack(uint2 v, float* f) { f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y); }
  __device__ static uint2 pack(const float* f) { return make_uint2(__float_as_uint(f[0]), __float_as_uint(f[1])); }
};

template <>
struct Unit<DT_BF16> {
  static constexpr int N = 4;
  __device__ static void unpack(uint2 v, float* f) {
    f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xffff0000u);
  }
  __device__ static uint2 pack(const float* f) {
    __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
    return make_uint2(*reinterpret_cast<unsigned int*>(&a), *reinterpret_cast<unsigned int*>(&b));
  }
};

template <>
struct Unit<DT_F16> {
  static constexpr int N = 4;
  __device__ static void unpack(uint2 v, float* f) {
    float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
  __device__ static uint2 pack(const float* f) {
    __half2 a = __floats2half2_rn(f[0], f[1]);
    __half2 b = __floats2half2_rn(f[2], f[3]);
    return make_uint2(*reinterpret_cast<unsigned int*>(&a), *reinterpret_cast<unsigned int*>(&b));
  }
};

template <int RED>
__device__ __forceinline__ float combine(float a, float b) {
  if (RED == RED_PROD) return a * b;
  if (RED == RED_MIN) return fminf(a, b);
  if (RED == RED_MAX) return fmaxf(a, b);
  return a + b;
}

__device__ void record_failure(const OneShotArgs& a, int code, int source, long long line) {
  if (atomicCAS(&a.control->status, ST_OK, code) == ST_OK) {
    a.control->detail[0] = a.rank;
    a.control->detail[1] = -2;        // the one-shot path (no device block)
    a.control->detail[2] = source;
    a.control->detail[3] = (int)line;
  }
  __threadfence();
}

// Wait until both halves of the line carry `tag`; false on timeout or abort.
__device__ __forceinline__ bool wait_line(const OneShotArgs& a, const char* p, unsigned int tag, uint2& d,
                                          int source, long long line) {
  unsigned long long lo, hi;
  ld_line(p, lo, hi);
  if ((unsigned int)(lo >> 32) == tag && (unsigned int)(hi >> 32) == tag) {
    d = make_uint2((unsigned int)lo, (unsigned int)hi);
    return true;
  }
  const unsigned long long t0 = globaltimer();
  unsigned int spins = 0;
  for (;;) {
    ld_line(p, lo, hi);
    if ((unsigned int)(lo >> 32) == tag && (unsigned int)(hi >> 32) == tag) break;
    if ((++spins & 255u) == 0) {
      if (ld_volatile_int(&a.control->abort_request) || ld_volatile_int(&a.control->status) != ST_OK) return false;
      if (globaltimer() - t0 > a.timeout_ns) {
        record_failure(a, ST_TIMEOUT, source, line);
        return false;
      }
    }
  }
  d = make_uint2((unsigned int)lo, (unsigned int)hi);
  return true;
}

template <int DT, int RED, int COLL>
__global__ void __launch_bounds__(kThreads) oneshot_kernel(OneShotArgs a) {
  using U = Unit<DT>;
  const unsigned long long seq = ld_volatile_u64(&a.control->ll_seq);
  const unsigned int tag = (unsigned int)(seq % 0xfffffffeull) + 1u;
  const long long half = (long long)a.nranks * a.ll_src_bytes;
  const long long region = a.ll_off + (long long)(seq & 1ull) * half;
  const long long units = a.bytes >> 3;
  const long long first = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const char* in = a.base[a.rank] + a.in_off;
  char* out = a.base[a.rank] + a.out_off;

  // push: this rank's lines into its source slot of every peer's region
  const long long slot = region + (long long)a.rank * a.ll_src_bytes;
  for (long long u = first; u < units; u += stride) {
    const uint2 d = ld_payload(in + u * 8);
    if (a.mc_base != nullptr) {
      mc_st_line(a.mc_base + slot + u * 16, d, tag);
    } else {
      for (int k = 1; k < a.nranks; ++k) {
        const int peer = (a.rank + k) % a.nranks;
        st_line(a.base[peer] + slot + u * 16, d, tag);
      }
    }
    if (COLL == OS_ALLGATHER) st_payload(out + ((long long)a.rank * units + u) * 8, d);
  }

  // receive: every peer's lines from the local region
  const char* local = a.base[a.rank] + region;
  bool ok = true;
  for (long long u = first; u < units && ok; u += stride) {
    if (COLL == OS_ALLGATHER) {
      for (int k = 1; k < a.nranks && ok; ++k) {
        const int src = (a.rank + k) % a.nranks;
        uint2 d;
        ok = wait_line(a, local + (long long)src * a.ll_src_bytes + u * 16, tag, d, src, u);
        if (ok) st_payload(out + ((long long)src * units + u) * 8, d);
      }
    } else {
      float acc[U::N], x[U::N];
      for (int src = 0; src < a.nranks && ok; ++src) {
        uint2 d;
        if (src == a.rank) {
          d = ld_payload(in + u * 8);
        } else {
          ok = wait_line(a, local + (long long)src * a.ll_src_bytes + u * 16, tag, d, src, u);
          if (!ok) break;
        }
        if (src == 0) {
          U::unpack(d, acc);
        } else {
          U::unpack(d, x);
#pragma unroll
          for (int e = 0; e < U::N; ++e) acc[e] = combine<RED>(acc[e], x[e]);
        }
      }
      if (!ok) break;
      if (a.do_scale) {
#pragma unroll
        for (int e = 0; e < U::N; ++e) acc[e] *= a.scale;
      }
      st_payload(out + u * 8, U::pack(acc));
    }
  }

  // the last CTA advances the launch counter for the next one-shot launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(&a.control->ll_arrive, 1u);
    if (prev == gridDim.x - 1) {
      a.control->ll_arrive = 0;
      a.control->ll_seq = seq + 1;
      __threadfence();
    }
  }
}

// Two-shot AllReduce for mid-size payloads: a reduce-scatter by LL lines (every rank pushes its part of
// slice j to rank j, which owns slice j = bytes/P), then an all-gather of the reduced slices by LL lines.
// Per GPU it moves about 4·bytes·(P−1)/P of lines instead of the one-shot's 2·bytes·(P−1), at the price of
// a second NVLink trip.  Both areas live in the launch's region half: the reduce-scatter area holds
// [P sources][2·slice] and the all-gather area after it [P owners][2·slice]; the half-reuse argument of the
// one-shot kernel applies to each area (a rank writes a half again only two launches later, after every
// peer has consumed it: its reduce-scatter lines after the owner's reduction of the previous launch that
// used the half, its all-gather lines after every rank's reduce-scatter push of the launch in between).
template <int DT, int RED>
__global__ void __launch_bounds__(kThreads) twoshot_kernel(OneShotArgs a) {
  using U = Unit<DT>;
  const unsigned long long seq = ld_volatile_u64(&a.control->ll_seq);
  const unsigned int tag = (unsigned int)(seq % 0xfffffffeull) + 1u;
  const long long half = (long long)a.nranks * a.ll_src_bytes;
  const long long region = a.ll_off + (long long)(seq & 1ull) * half;
  const long long su = (a.bytes / a.nranks) >> 3;          // 8-byte units of one owner slice
  const long long lines = su * 16;                          // line bytes of one source (or owner) per area
  const long long rs = region, ag = region + (long long)a.nranks * lines;
  const long long first = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const char* in = a.base[a.rank] + a.in_off;
  char* out = a.base[a.rank] + a.out_off;
  const char* local = a.base[a.rank];

  // 1. reduce-scatter push: this rank's part of every other owner's slice
  for (long long u = first; u < su; u += stride)
    for (int k = 1; k < a.nranks; ++k) {
      const int j = (a.rank + k) % a.nranks;
      const uint2 d = ld_payload(in + ((long long)j * su + u) * 8);
      st_line(a.base[j] + rs + (long long)a.rank * lines + u * 16, d, tag);
    }

  // 2. reduce the owned slice in rank order, 3. push the result to every rank
  bool ok = true;
  for (long long u = first; u < su && ok; u += stride) {
    float acc[U::N], x[U::N];
    for (int src = 0; src < a.nranks && ok; ++src) {
      uint2 d;
      if (src == a.rank) {
        d = ld_payload(in + ((long long)a.rank * su + u) * 8);
      } else {
        ok = wait_line(a, local + rs + (long long)src * lines + u * 16, tag, d, src, u);
        if (!ok) break;
      }
      if (src == 0) {
        U::unpack(d, acc);
      } else {
        U::unpack(d, x);
#pragma unroll
        for (int e = 0; e < U::N; ++e) acc[e] = combine<RED>(acc[e], x[e]);
      }
    }
    if (!ok) break;
    if (a.do_scale) {
#pragma unroll
      for (int e = 0; e < U::N; ++e) acc[e] *= a.scale;
    }
    const uint2 r = U::pack(acc);
    st_payload(out + ((long long)a.rank * su + u) * 8, r);
    const long long slot = ag + (long long)a.rank * lines + u * 16;
    if (a.mc_base != nullptr) {
      mc_st_line(a.mc_base + slot, r, tag);
    } else {
      for (int k = 1; k < a.nranks; ++k) st_line(a.base[(a.rank + k) % a.nranks] + slot, r, tag);
    }
  }

  // 4. the other owners' reduced slices
  for (long long u = first; u < su && ok; u += stride)
    for (int k = 1; k < a.nranks && ok; ++k) {
      const int j = (a.rank + k) % a.nranks;
      uint2 d;
      ok = wait_line(a, local + ag + (long long)j * lines + u * 16, tag, d, j, u);
      if (ok) st_payload(out + ((long long)j * su + u) * 8, d);
    }

  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(&a.control->ll_arrive, 1u);
    if (prev == gridDim.x - 1) {
      a.control->ll_arrive = 0;
      a.control->ll_seq = seq + 1;
      __threadfence();
    }
  }
}

template <int DT, int RED>
cudaError_t launch_coll(const OneShotArgs& a, dim3 grid, cudaStream_t stream) {
  void* args[] = {const_cast<OneShotArgs*>(&a)};
  if (a.coll == OS_ALLREDUCE_TWOSHOT)
    return cudaLaunchCooperativeKernel((void*)twoshot_kernel<DT, RED>, grid, dim3(kThreads), args, 0, stream);
  if (a.coll == OS_ALLGATHER)
    return cudaLaunchCooperativeKernel((void*)oneshot_kernel<DT, RED, OS_ALLGATHER>, grid, dim3(kThreads), args, 0,
                                       stream);
  return cudaLaunchCooperativeKernel((void*)oneshot_kernel<DT, RED, OS_ALLREDUCE>, grid, dim3(kThreads), args, 0,
                                     stream);
}

template <int DT>
cudaError_t launch_dt(const OneShotArgs& a, dim3 grid, cudaStream_t stream) {
  switch (a.redop) {
    case RED_PROD: return launch_coll<DT, RED_PROD>(a, grid, stream);
    case RED_MIN: return launch_coll<DT, RED_MIN>(a, grid, stream);
    case RED_MAX: return launch_coll<DT, RED_MAX>(a, grid, stream);
    default: return launch_coll<DT, RED_SUM>(a, grid, stream);
  }
}

}  // namespace

long long oneshot_region_bytes(int nranks, long long max_bytes) {
  const long long src = ((max_bytes + 7) / 8) * 16;
  return 2ll * nranks * src;
}

int oneshot_max_ctas() {
  static int cached[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  int sms = 0, per_sm = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, oneshot_kernel<DT_F32, RED_SUM, OS_ALLREDUCE>, kThreads, 0);
  int b = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, oneshot_kernel<DT_BF16, RED_SUM, OS_ALLREDUCE>, kThreads, 0);
  if (b < per_sm) per_sm = b;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, twoshot_kernel<DT_BF16, RED_SUM>, kThreads, 0);
  if (b < per_sm) per_sm = b;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, twoshot_kernel<DT_F32, RED_SUM>, kThreads, 0);
  if (b < per_sm) per_sm = b;
  const int v = sms * (per_sm < 1 ? 1 : per_sm);
  if (dev >= 0 && dev < 64) cached[dev] = v;
  return v;
}

cudaError_t launch_oneshot(const OneShotArgs& a, cudaStream_t stream) {
  if (a.nranks < 1 || a.nranks > kMaxRanks || a.rank < 0 || a.rank >= a.nranks) return cudaErrorInvalidValue;
  if (a.in_off % 8 || a.out_off % 8 || a.ll_off % 16 || a.ll_src_bytes % 16) return cudaErrorInvalidValue;
  if (a.coll == OS_ALLREDUCE_TWOSHOT) {
    // both areas (4·bytes of lines) must fit the region half
    if (a.bytes <= 0 || a.bytes % (8ll * a.nranks) || 4 * a.bytes > (long long)a.nranks * a.ll_src_bytes)
      return cudaErrorInvalidValue;
  } else if (a.bytes <= 0 || a.bytes % 8 || a.ll_src_bytes < 2 * a.bytes) {
    return cudaErrorInvalidValue;
  }
  const long long units = a.coll == OS_ALLREDUCE_TWOSHOT ? a.bytes / 8 / a.nranks : a.bytes / 8;
  long long ctas = (units + kThreads - 1) / kThreads;
  const int cap = oneshot_max_ctas();
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  dim3 grid((unsigned)ctas);
  switch (a.dtype) {
    case DT_F32: return launch_dt<DT_F32>(a, grid, stream);
    case DT_BF16: return launch_dt<DT_BF16>(a, grid, stream);
    case DT_F16: return launch_dt<DT_F16>(a, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vb

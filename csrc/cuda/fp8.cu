// Block-scaled FP8 (e4m3) payloads for AllGather.
//
// quantize: every block of `block` elements gets one fp32 scale
// amax(block) / 448 (the largest finite e4m3 value) and its elements are
// stored as e4m3 of x / scale (round to nearest even, saturating);
// dequantize: x = e4m3 * scale.  A gathered payload is [fp8 bytes | fp32
// scales] per rank, so an AllGather moves about a quarter (fp32 input) or a
// half (bf16 input) of the bytes.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "vb/launch.h"

namespace vb {
namespace {

__device__ __forceinline__ float load_f(const void* p, long long i, int dt) {
  if (dt == DT_F32) return static_cast<const float*>(p)[i];
  if (dt == DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void store_f(void* p, long long i, int dt, float v) {
  if (dt == DT_F32) static_cast<float*>(p)[i] = v;
  else if (dt == DT_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}

// one warp per block of elements
__global__ void quantize_kernel(const void* in, unsigned char* q, float* scales, long long n, int block, int dt) {
  const int lane = threadIdx.x & 31;
  const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nblocks = (n + block - 1) / block;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long b = warp; b < nblocks; b += warps) {
    const long long lo = b * block;
    const long long hi = lo + block < n ? lo + block : n;
    float amax = 0.f;
    for (long long i = lo + lane; i < hi; i += 32) amax = fmaxf(amax, fabsf(load_f(in, i, dt)));
    for (int off = 16; off; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float scale = amax > 0.f ? amax / 448.f : 1.f;
    const float inv = 1.f / scale;
    if (lane == 0) scales[b] = scale;
    for (long long i = lo + lane; i < hi; i += 32) {
      __nv_fp8_e4m3 v(load_f(in, i, dt) * inv);
      q[i] = *reinterpret_cast<unsigned char*>(&v);
    }
  }
}

__global__ void dequantize_kernel(const unsigned char* q, const float* scales, void* out, long long n, int block,
                                  int dt) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    __nv_fp8_e4m3 v;
    *reinterpret_cast<unsigned char*>(&v) = q[i];
    store_f(out, i, dt, float(v) * scales[i / block]);
  }
}

// ---- fused AllGather ------------------------------------------------------------------------------
//
// Layout of one staging parity for n elements: e4m3 bytes [0, pad16(n)), then one fp32 scale per 128
// elements [pad16(n), pad16(n) + pad16(4 * ceil(n / 128))).  Launch k uses parity k & 1.
//
// Work split: the n elements form groups of 16 (one 16-byte e4m3 vector per lane); CTA c owns the
// groups [c * G / ctas, (c + 1) * G / ctas) of EVERY rank's chunk, rounded to whole 128-element blocks so
// a block's scale is computed by the CTA that owns it.  Phase A: CTA c quantizes its groups of this
// rank's input into the staging parity and writes their dequantized values into this rank's part of
// the output, then publishes flag[c] = k + 1 (st.release.sys after a CTA barrier).  Phase B: for every
// peer q (rank + 1, rank + 2, ...) CTA c waits until q's flag[c] >= k + 1 (ld.acquire.sys, bounded by
// %globaltimer), then loads q's staged groups over NVLink and dequantizes them into part q of the
// output.  Reuse of a staging parity is safe without any further wait: rank r rewrites parity k & 1 in
// launch k + 2, and it cannot start that launch before its launch k + 1 saw every peer's flags of k + 1,
// which each peer raises only in its launch k + 1, i.e. after its launch k (and all of its reads of
// r's parity k & 1) has finished.
constexpr int kFp8Threads = 256;
constexpr int kFp8Block = 128;                   // elements per scale
constexpr int kGroupsPerBlock = kFp8Block / 16;  // 8 lanes share one block

__device__ __forceinline__ unsigned long long fp8_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long fp8_ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fp8_st_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint4 fp8_ld_peer(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ long long pad16(long long b) { return (b + 15) / 16 * 16; }

// 16 consecutive input elements of group g as floats
template <int DT>
__device__ __forceinline__ void load16(const void* in, long long g, float* f) {
  if (DT == DT_F32) {
    const float4* p = reinterpret_cast<const float4*>(in) + g * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float4 v = p[i];
      f[4 * i] = v.x; f[4 * i + 1] = v.y; f[4 * i + 2] = v.z; f[4 * i + 3] = v.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(in) + g * 2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 v = p[i];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (DT == DT_BF16) {
          f[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
          f[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
        } else {
          float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          f[8 * i + 2 * j] = x.x;
          f[8 * i + 2 * j + 1] = x.y;
        }
      }
    }
  }
}

template <int DT>
__device__ __forceinline__ void store16(void* out, long long g, const float* f) {
  if (DT == DT_F32) {
    float4* p = reinterpret_cast<float4*>(out) + g * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = make_float4(f[4 * i], f[4 * i + 1], f[4 * i + 2], f[4 * i + 3]);
  } else {
    uint4* p = reinterpret_cast<uint4*>(out) + g * 2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (DT == DT_BF16) {
          __nv_bfloat162 h = __floats2bfloat162_rn(f[8 * i + 2 * j], f[8 * i + 2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(f[8 * i + 2 * j], f[8 * i + 2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      p[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

__device__ __forceinline__ uint4 encode16(const float* f, float inv) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      __nv_fp8_e4m3 v(f[4 * j + b] * inv);
      word |= (uint32_t)(*reinterpret_cast<unsigned char*>(&v)) << (8 * b);
    }
    w[j] = word;
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void decode16(const uint4& v, float scale, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      __nv_fp8_e4m3 x;
      *reinterpret_cast<unsigned char*>(&x) = (unsigned char)(w[j] >> (8 * b));
      f[4 * j + b] = float(x) * scale;
    }
  }
}

__device__ void fp8_fail(const Fp8AgArgs& a, int code, int peer) {
  if (atomicCAS(&a.control->status, ST_OK, code) == ST_OK) {
    a.control->detail[0] = a.rank;
    a.control->detail[1] = peer;
    a.control->detail[2] = blockIdx.x;
    a.control->detail[3] = -1;
  }
  __threadfence();
}

template <int DT>
__global__ void __launch_bounds__(kFp8Threads) fp8_allgather_kernel(const Fp8AgArgs a) {
  __shared__ unsigned long long s_seq;
  __shared__ int s_stop;
  if (threadIdx.x == 0) {
    s_seq = *(volatile unsigned long long*)&a.control->fp8_seq;
    s_stop = 0;
  }
  __syncthreads();
  const unsigned long long seq = s_seq;
  const long long groups = a.n / 16;
  const long long blocks = (a.n + kFp8Block - 1) / kFp8Block;
  const long long stage = pad16(a.n) + pad16(4 * blocks);   // equals fp8_stage_bytes(n)
  const long long par_off = a.stage_off + (long long)(seq & 1ull) * stage;
  // this CTA's groups, whole blocks only
  const long long b0 = blocks * blockIdx.x / a.ctas, b1 = blocks * (blockIdx.x + 1) / a.ctas;
  const long long g0 = b0 * kGroupsPerBlock, g1 = min(groups, b1 * kGroupsPerBlock);
  const int lane = threadIdx.x & 31;
  const long long esize = DT == DT_F32 ? 4 : 2;
  char* my_stage = a.base[a.rank] + par_off;
  char* out = static_cast<char*>(a.out);
  // ---- phase A: quantize this rank's groups, write their dequantized values into our own part.  Each thread
  // loads two groups (kFp8Threads apart) before it works on either, so twice the input is in flight.
  constexpr int UA = 2;
  for (long long base = g0 + (threadIdx.x & ~31); base < g1; base += (long long)UA * kFp8Threads) {
    float f[UA][16];
    bool live[UA];
#pragma unroll
    for (int u = 0; u < UA; ++u) {
      const long long g = base + (long long)u * kFp8Threads + lane;
      live[u] = g < g1;
      if (live[u]) load16<DT>(a.in, g, f[u]);
    }
#pragma unroll
    for (int u = 0; u < UA; ++u) {
      const long long g = base + (long long)u * kFp8Threads + lane;
      float amax = 0.f;
      if (live[u]) {
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(f[u][i]));
      }
      // the 8 lanes of one 128-element block (aligned: base is a multiple of 32 groups, and so is
      // u * kFp8Threads) share its amax; every lane of the warp takes part in the shuffles
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      const float scale = amax > 0.f ? amax / 448.f : 1.f;
      if (live[u]) {
        const uint4 q = encode16(f[u], 1.f / scale);
        *reinterpret_cast<uint4*>(my_stage + g * 16) = q;
        if ((g % kGroupsPerBlock) == 0)
          reinterpret_cast<float*>(my_stage + pad16(a.n))[g / kGroupsPerBlock] = scale;
        decode16(q, scale, f[u]);
        store16<DT>(out + (long long)a.rank * a.n * esize, g, f[u]);
      }
    }
  }
  __syncthreads();
  unsigned long long* flags = reinterpret_cast<unsigned long long*>(a.base[a.rank] + a.flag_off);
  if (threadIdx.x == 0) fp8_st_release(flags + blockIdx.x, seq + 1);
  // ---- phase B: every peer's staged groups of this CTA's range, dequantized into part q
  for (int step = 1; step < a.nranks; ++step) {
    const int q = (a.rank + step) % a.nranks;
    if (threadIdx.x == 0) {
      const unsigned long long* f = reinterpret_cast<const unsigned long long*>(a.base[q] + a.flag_off) + blockIdx.x;
      if (fp8_ld_acquire(f) < seq + 1) {
        const unsigned long long t0 = fp8_timer();
        unsigned int spins = 0;
        while (fp8_ld_acquire(f) < seq + 1) {
          if ((++spins & 63u) == 0) {
            if (*(volatile int*)&a.control->status != ST_OK || *(volatile int*)&a.control->abort_request) {
              s_stop = 1;
              break;
            }
            if (fp8_timer() - t0 > a.timeout_ns) {
              fp8_fail(a, ST_TIMEOUT, q);
              s_stop = 1;
              break;
            }
          }
        }
      }
    }
    __syncthreads();
    if (s_stop) break;
    const char* peer_stage = a.base[q] + par_off;
    const float* peer_scales = reinterpret_cast<const float*>(peer_stage + pad16(a.n));
    char* part = out + (long long)q * a.n * esize;
    // four 16-byte loads per thread in flight before any is decoded
    constexpr int U = 4;
    for (long long g = g0 + threadIdx.x; g < g1; g += (long long)U * kFp8Threads) {
      uint4 v[U];
      float sc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long gu = g + (long long)u * kFp8Threads;
        if (gu < g1) {
          v[u] = fp8_ld_peer(peer_stage + gu * 16);
          sc[u] = peer_scales[gu / kGroupsPerBlock];
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long gu = g + (long long)u * kFp8Threads;
        if (gu < g1) {
          float f[16];
          decode16(v[u], sc[u], f);
          store16<DT>(part, gu, f);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.control->fp8_arrive, 1u) == gridDim.x - 1) {
      a.control->fp8_arrive = 0;
      a.control->fp8_seq = seq + 1;
      __threadfence();
    }
  }
}

int grid_for(long long work) {
  long long g = (work + 255) / 256;
  return (int)(g > 4096 ? 4096 : (g < 1 ? 1 : g));
}

}  // namespace

cudaError_t launch_quantize_fp8(const void* in, unsigned char* q, float* scales, long long n, int block, int dtype,
                                cudaStream_t stream) {
  long long nblocks = (n + block - 1) / block;
  quantize_kernel<<<grid_for(nblocks * 32), 256, 0, stream>>>(in, q, scales, n, block, dtype);
  return cudaGetLastError();
}

cudaError_t launch_dequantize_fp8(const unsigned char* q, const float* scales, void* out, long long n, int block,
                                  int dtype, cudaStream_t stream) {
  dequantize_kernel<<<grid_for(n), 256, 0, stream>>>(q, scales, out, n, block, dtype);
  return cudaGetLastError();
}

long long fp8_stage_bytes(long long n) {
  return (n + 15) / 16 * 16 + (4 * ((n + kFp8Block - 1) / kFp8Block) + 15) / 16 * 16;
}

int fp8_allgather_max_ctas() {
  static int cached[64] = {};
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) return cached[dev];
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int lo = 1 << 30;
  const void* fns[] = {(const void*)fp8_allgather_kernel<DT_F32>, (const void*)fp8_allgather_kernel<DT_BF16>,
                       (const void*)fp8_allgather_kernel<DT_F16>};
  for (const void* fn : fns) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kFp8Threads, 0) == cudaSuccess && per_sm < lo)
      lo = per_sm;
  }
  const int v = sms * (lo == (1 << 30) ? 0 : lo);
  if (dev >= 0 && dev < 64) cached[dev] = v;
  return v;
}

cudaError_t launch_fp8_allgather(const Fp8AgArgs& a, cudaStream_t stream) {
  if (a.n <= 0 || a.n % 16 || a.ctas < 1 || a.nranks < 1 || a.nranks > kMaxRanks || a.rank < 0 ||
      a.rank >= a.nranks || a.ctas > fp8_allgather_max_ctas())
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.in) | reinterpret_cast<uintptr_t>(a.out)) % 16 || a.stage_off % 16 ||
      a.flag_off % 8)
    return cudaErrorMisalignedAddress;
  void* args[] = {const_cast<Fp8AgArgs*>(&a)};
  dim3 grid(a.ctas), block(kFp8Threads);
  // co-residency of every CTA: peers' CTAs wait on this rank's CTAs of the same index
  switch (a.dtype) {
    case DT_F32: return cudaLaunchCooperativeKernel((void*)fp8_allgather_kernel<DT_F32>, grid, block, args, 0, stream);
    case DT_BF16: return cudaLaunchCooperativeKernel((void*)fp8_allgather_kernel<DT_BF16>, grid, block, args, 0, stream);
    case DT_F16: return cudaLaunchCooperativeKernel((void*)fp8_allgather_kernel<DT_F16>, grid, block, args, 0, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vb

// Calibration probes: device-timed primitive kernels.
//
// copy  — dst = src (local copy, or a remote pull/push when one side is a
//         peer-mapped address): the send / recv primitives of the cost model;
// reduce — dst = src0 + ... + src{k-1} in fp32 (local reduce, or a receive-
//         reduce-copy when a source is remote).
// The host times them with CUDA events and fits α/β per component.
#include <cuda_runtime.h>

#include "vb/launch.h"

namespace vb {
namespace {

__device__ __forceinline__ uint4 ldv(const char* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void stv(char* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

template <int U>
__global__ void __launch_bounds__(512) copy_probe(char* dst, const char* src, long long nvec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long v0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; v0 < nvec; v0 += stride * U) {
    uint4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v0 + u * stride < nvec) r[u] = ldv(src + (v0 + u * stride) * 16);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v0 + u * stride < nvec) stv(dst + (v0 + u * stride) * 16, r[u]);
  }
}

struct Srcs {
  const char* p[8];
};

__global__ void __launch_bounds__(512) reduce_probe(char* dst, Srcs s, int k, long long nvec) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < nvec; v += stride) {
    uint4 r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < k) r[i] = ldv(s.p[i] + v * 16);
    float acc[4] = {__uint_as_float(r[0].x), __uint_as_float(r[0].y), __uint_as_float(r[0].z), __uint_as_float(r[0].w)};
#pragma unroll
    for (int i = 1; i < 8; ++i)
      if (i < k) {
        acc[0] += __uint_as_float(r[i].x); acc[1] += __uint_as_float(r[i].y);
        acc[2] += __uint_as_float(r[i].z); acc[3] += __uint_as_float(r[i].w);
      }
    stv(dst + v * 16, make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                                 __float_as_uint(acc[3])));
  }
}

}  // namespace

cudaError_t launch_copy_probe(void* dst, const void* src, long long bytes, int ctas, int threads, int unroll,
                              cudaStream_t stream) {
  long long nvec = bytes / 16;
  switch (unroll) {
    case 1: copy_probe<1><<<ctas, threads, 0, stream>>>((char*)dst, (const char*)src, nvec); break;
    case 2: copy_probe<2><<<ctas, threads, 0, stream>>>((char*)dst, (const char*)src, nvec); break;
    case 8: copy_probe<8><<<ctas, threads, 0, stream>>>((char*)dst, (const char*)src, nvec); break;
    default: copy_probe<4><<<ctas, threads, 0, stream>>>((char*)dst, (const char*)src, nvec); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_reduce_probe(void* dst, const void* const* srcs, int k, long long bytes, int ctas, int threads,
                                cudaStream_t stream) {
  if (k < 1 || k > 8) return cudaErrorInvalidValue;
  Srcs s = {};
  for (int i = 0; i < k; ++i) s.p[i] = (const char*)srcs[i];
  reduce_probe<<<ctas, threads, 0, stream>>>((char*)dst, s, k, bytes / 16);
  return cudaGetLastError();
}

}  // namespace vb

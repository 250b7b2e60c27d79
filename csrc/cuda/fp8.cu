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

}  // namespace vb

// Small helper kernels: deterministic fills, a standalone scale pass (the
// unfused baseline of the reference's post-collective average), an analytic
// output checker, a 2D pitched copy (staging of strided tensors; the
// reference's stride copy is
// third_party/msccl/src/collectives/device/stride_copy.cu:6-25) and a
// %globaltimer reader.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "vb/launch.h"

namespace vb {
namespace {

__device__ __forceinline__ float ld_elem(const void* p, long long i, int dt) {
  if (dt == DT_F32) return static_cast<const float*>(p)[i];
  if (dt == DT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void st_elem(void* p, long long i, int dt, float v) {
  if (dt == DT_F32) static_cast<float*>(p)[i] = v;
  else if (dt == DT_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}

// Pattern 0: value = 1 + ((3*rank + i) mod 5), the analytic pattern of the
// reference driver (runtime/execution/gpu_operations.cu); pattern 1: a
// counter-based hash mapped to [-1, 1).
__device__ __forceinline__ float pattern_value(int pattern, int rank, long long i, unsigned long long seed) {
  if (pattern == 0) return 1.0f + (float)((3 * rank + i) % 5);
  unsigned long long x = seed ^ ((unsigned long long)rank << 40) ^ (unsigned long long)i * 0x9E3779B97F4A7C15ull;
  x ^= x >> 33; x *= 0xff51afd7ed558ccdull; x ^= x >> 33; x *= 0xc4ceb9fe1a85ec53ull; x ^= x >> 33;
  return (float)((x >> 40) & 0xffffff) / 8388608.0f - 1.0f;
}

__global__ void fill_kernel(void* dst, long long n, int dt, int pattern, int rank, unsigned long long seed) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    st_elem(dst, i, dt, pattern_value(pattern, rank, i, seed));
}

__global__ void scale_kernel(void* dst, const void* src, long long n, int dt, float scale) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    st_elem(dst, i, dt, ld_elem(src, i, dt) * scale);
}

// Analytic value of pattern 0 and the fp64 reduction of it over all ranks.
__device__ __forceinline__ double pattern0(int rank, long long i) { return 1.0 + (double)((3 * rank + i) % 5); }

__device__ double reduced0(long long i, int nranks, int redop) {
  double acc = 0;
  for (int r = 0; r < nranks; ++r) {
    double v = pattern0(r, i);
    if (r == 0) acc = v;
    else if (redop == RED_PROD) acc *= v;
    else if (redop == RED_MIN) acc = acc < v ? acc : v;
    else if (redop == RED_MAX) acc = acc > v ? acc : v;
    else acc += v;
  }
  return acc;
}

// Checks, in fp64, the output of a collective whose inputs follow pattern 0.
// coll: 0 allreduce, 1 allgather, 2 reduce_scatter, 3 broadcast (root's input),
// 4 reduce (the reduction, on the root), 5 alltoall (part s of rank r is part r
// of rank s), 6 this rank's own input (a read-only re-check).  ``count`` is the
// input elements per rank; reductions are multiplied by ``scale``.
__global__ void check_kernel(const void* out, long long n, int dt, int coll, int redop, int nranks, int rank,
                             long long count, double atol, double rtol, unsigned long long* bad, int root,
                             double scale) {
  unsigned long long local = 0;
  const long long part = nranks > 0 ? count / nranks : count;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    double expect;
    switch (coll) {
      case 1: expect = pattern0((int)(i / count), i % count); break;
      case 2: expect = reduced0((long long)rank * part + i, nranks, redop) * scale; break;
      case 3: expect = pattern0(root, i); break;
      case 5: expect = pattern0((int)(i / part), (long long)rank * part + i % part); break;
      case 6: expect = pattern0(rank, i); break;
      default: expect = reduced0(i, nranks, redop) * scale; break;   // 0 allreduce, 4 reduce
    }
    double got = ld_elem(out, i, dt);
    double err = got - expect;
    if (err < 0) err = -err;
    if (!(err <= atol + rtol * (expect < 0 ? -expect : expect))) ++local;
  }
  if (local) atomicAdd(bad, local);
}

__global__ void timer_kernel(unsigned long long* dst) {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  *dst = t;
}

// 2D pitched copy: row r of ``rows`` rows of ``row_bytes`` bytes moves from
// src + r*src_pitch to dst + r*dst_pitch.  V is the widest access that every
// address, pitch and row length allows (16, 8, 4 or 1 bytes); the flat index
// over (row, unit) is grid-strided so any shape fills the grid.
template <typename V>
__global__ void strided_copy_kernel(char* dst, long long dst_pitch, const char* src, long long src_pitch,
                                    long long units_per_row, long long total) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / units_per_row, c = i - r * units_per_row;
    *reinterpret_cast<V*>(dst + r * dst_pitch + c * (long long)sizeof(V)) =
        *reinterpret_cast<const V*>(src + r * src_pitch + c * (long long)sizeof(V));
  }
}

int grid_for(long long n) {
  long long g = (n + 255) / 256;
  return (int)(g > 4096 ? 4096 : (g < 1 ? 1 : g));
}

}  // namespace

cudaError_t launch_fill(void* dst, long long n, int dtype, int pattern, int rank, unsigned long long seed,
                        cudaStream_t stream) {
  fill_kernel<<<grid_for(n), 256, 0, stream>>>(dst, n, dtype, pattern, rank, seed);
  return cudaGetLastError();
}

cudaError_t launch_scale(void* dst, const void* src, long long n, int dtype, float scale, cudaStream_t stream) {
  scale_kernel<<<grid_for(n), 256, 0, stream>>>(dst, src, n, dtype, scale);
  return cudaGetLastError();
}

cudaError_t launch_check(const void* out, long long n, int dtype, int collective, int redop, int nranks, int rank,
                         long long count_per_rank, double atol, double rtol, unsigned long long* bad,
                         cudaStream_t stream, int root, double scale) {
  if (n <= 0) return cudaSuccess;
  check_kernel<<<grid_for(n), 256, 0, stream>>>(out, n, dtype, collective, redop, nranks, rank, count_per_rank, atol,
                                               rtol, bad, root, scale);
  return cudaGetLastError();
}

cudaError_t launch_strided_copy(void* dst, long long dst_pitch, const void* src, long long src_pitch,
                                long long row_bytes, long long rows, cudaStream_t stream) {
  if (rows <= 0 || row_bytes <= 0) return cudaSuccess;
  if (row_bytes > dst_pitch && rows > 1) return cudaErrorInvalidValue;
  if (row_bytes > src_pitch && rows > 1) return cudaErrorInvalidValue;
  unsigned long long bits = reinterpret_cast<unsigned long long>(dst) | reinterpret_cast<unsigned long long>(src) |
                            (unsigned long long)dst_pitch | (unsigned long long)src_pitch |
                            (unsigned long long)row_bytes;
  int width = (bits % 16 == 0) ? 16 : (bits % 8 == 0) ? 8 : (bits % 4 == 0) ? 4 : 1;
  long long units = row_bytes / width, total = units * rows;
  // at most 8 resident 256-thread blocks on each of the 148 SMs; fewer when there is less work
  long long blocks = (total + 255) / 256;
  int grid = (int)(blocks > 148 * 8 ? 148 * 8 : blocks);
  char* d = static_cast<char*>(dst);
  const char* sp = static_cast<const char*>(src);
  if (width == 16) strided_copy_kernel<uint4><<<grid, 256, 0, stream>>>(d, dst_pitch, sp, src_pitch, units, total);
  else if (width == 8) strided_copy_kernel<uint2><<<grid, 256, 0, stream>>>(d, dst_pitch, sp, src_pitch, units, total);
  else if (width == 4) strided_copy_kernel<unsigned int><<<grid, 256, 0, stream>>>(d, dst_pitch, sp, src_pitch, units,
                                                                                    total);
  else strided_copy_kernel<unsigned char><<<grid, 256, 0, stream>>>(d, dst_pitch, sp, src_pitch, units, total);
  return cudaGetLastError();
}

cudaError_t launch_read_timer(unsigned long long* dst, cudaStream_t stream) {
  timer_kernel<<<1, 1, 0, stream>>>(dst);
  return cudaGetLastError();
}

}  // namespace vb

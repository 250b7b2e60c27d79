// Persistent schedule interpreter for sm_100a.
//
// One CTA per (device block, lane).  A CTA walks its block's steps for every
// pipeline iteration; each data step moves the CTA's piece of one or more
// chunks from local or peer-mapped memory (NVLink through NVSwitch) — with
// 16-byte vector loads, or, in the staged instances, with TMA bulk copies into
// shared memory — combines sources in fp32, applies the fused scale and
// stores once (NVLS steps use multimem.ld_reduce / multimem.st instead).  Ordering uses 64-bit monotone flags in the symmetric heap:
// waits poll with ld.acquire.sys (warp 0, one wait per lane), publications
// use st.release.sys after a CTA barrier.  Every wait is bounded by a
// %globaltimer deadline; on expiry the CTA records the failure in the
// control block's status word, which the other CTAs' waits poll and stop on,
// and returns, so a broken schedule or a missing peer never hangs the GPU.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "vb/launch.h"

namespace vb {
namespace {

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ int ld_volatile_int(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_vec(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// the same load with an L2 prefetch hint: the L2 fetches the whole 256-byte block around the address
__device__ __forceinline__ uint4 ld_vec_pf(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_vec(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// NVLS multimem: the switch reduces the 16 bytes at this offset over every
// GPU bound to the multicast object, or replicates a store to all of them.
template <int DT>
__device__ __forceinline__ uint4 mc_ld_reduce(const char* p);

template <>
__device__ __forceinline__ uint4 mc_ld_reduce<DT_F32>(const char* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}

template <>
__device__ __forceinline__ uint4 mc_ld_reduce<DT_BF16>(const char* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}

template <>
__device__ __forceinline__ uint4 mc_ld_reduce<DT_F16>(const char* p) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mc_st(char* p, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w) : "memory");
}

// ---- TMA bulk staging (cp.async.bulk + mbarrier) ---------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 state;\n mbarrier.arrive.expect_tx.shared::cta.b64 state, [%0], %1;\n}"
               ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done) : "r"(bar), "r"(parity) : "memory");
  return done != 0;
}

// global (local or peer-mapped, 16-byte aligned) -> shared, completion counted on `bar`
__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst_smem), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// shared -> this GPU's global memory (16-byte aligned, a multiple of 16 bytes), one bulk group per call
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n"
               "cp.async.bulk.commit_group;" ::"l"(dst), "r"(src_smem), "r"(bytes) : "memory");
}

// the issuing thread's bulk stores have read their shared-memory sources
__device__ __forceinline__ void bulk_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// the issuing thread's bulk stores are complete, and ordered before its later generic-proxy accesses
__device__ __forceinline__ void bulk_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;\n"
               "fence.proxy.async.global;" ::: "memory");
}

template <int DT>
struct VecT;

template <>
struct VecT<DT_F32> {
  static constexpr int N = 4;
  __device__ static void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  }
  __device__ static uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};

template <>
struct VecT<DT_BF16> {
  static constexpr int N = 8;
  __device__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ static uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

template <>
struct VecT<DT_F16> {
  static constexpr int N = 8;
  __device__ static void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 x = __half22float2(h);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
  __device__ static uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

template <int RED>
__device__ __forceinline__ float combine(float a, float b) {
  if (RED == RED_PROD) return a * b;
  if (RED == RED_MIN) return fminf(a, b);
  if (RED == RED_MAX) return fmaxf(a, b);
  return a + b;
}

// Move one piece: dst[v] = scale? * op(src0[v], ..., src_{K-1}[v]) for vectors v in [0, nvec).
// K is a compile-time source count so that all K*U loads of a thread are in flight together.
template <int DT, int RED, int K, int U, bool PF = false>
__device__ __forceinline__ void move_fixed(char* dst, const char* const* src, long long nvec, bool do_scale,
                                           float scale) {
  using V = VecT<DT>;
  const long long stride = (long long)blockDim.x * U;
  for (long long v0 = threadIdx.x; v0 < nvec; v0 += stride) {
    uint4 raw[K][U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      long long v = v0 + (long long)u * blockDim.x;
      if (v < nvec) {
#pragma unroll
        for (int k = 0; k < K; ++k) raw[k][u] = PF ? ld_vec_pf(src[k] + v * 16) : ld_vec(src[k] + v * 16);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      long long v = v0 + (long long)u * blockDim.x;
      if (v >= nvec) continue;
      if (K == 1 && !do_scale) {
        st_vec(dst + v * 16, raw[0][u]);
        continue;
      }
      float acc[V::N], tmp[V::N];
      V::unpack(raw[0][u], acc);
#pragma unroll
      for (int k = 1; k < K; ++k) {
        V::unpack(raw[k][u], tmp);
#pragma unroll
        for (int e = 0; e < V::N; ++e) acc[e] = combine<RED>(acc[e], tmp[e]);
      }
      if (do_scale) {
#pragma unroll
        for (int e = 0; e < V::N; ++e) acc[e] *= scale;
      }
      st_vec(dst + v * 16, V::pack(acc));
    }
  }
}

// Any source count: accumulate source by source (used for K > 8).
template <int DT, int RED>
__device__ void move_generic(char* dst, const char* const* src, int nsrc, long long nvec, bool do_scale,
                             float scale) {
  using V = VecT<DT>;
  for (long long v = threadIdx.x; v < nvec; v += blockDim.x) {
    float acc[V::N], tmp[V::N];
    V::unpack(ld_vec(src[0] + v * 16), acc);
    for (int k = 1; k < nsrc; ++k) {
      V::unpack(ld_vec(src[k] + v * 16), tmp);
#pragma unroll
      for (int e = 0; e < V::N; ++e) acc[e] = combine<RED>(acc[e], tmp[e]);
    }
    if (do_scale)
#pragma unroll
      for (int e = 0; e < V::N; ++e) acc[e] *= scale;
    st_vec(dst + v * 16, V::pack(acc));
  }
}

// dst(all ranks) = scale? * sum over ranks of src, through the multicast addresses.
template <int DT, int U>
__device__ void mc_allreduce_piece(char* mc_dst, const char* mc_src, long long nvec, bool do_scale, float scale) {
  using V = VecT<DT>;
  const long long stride = (long long)blockDim.x * U;
  for (long long v0 = threadIdx.x; v0 < nvec; v0 += stride) {
    uint4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      long long v = v0 + (long long)u * blockDim.x;
      if (v < nvec) r[u] = mc_ld_reduce<DT>(mc_src + v * 16);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      long long v = v0 + (long long)u * blockDim.x;
      if (v >= nvec) continue;
      uint4 out = r[u];
      if (do_scale) {
        float f[V::N];
        V::unpack(r[u], f);
#pragma unroll
        for (int e = 0; e < V::N; ++e) f[e] *= scale;
        out = V::pack(f);
      }
      mc_st(mc_dst + v * 16, out);
    }
  }
}

// dst(all ranks) = src(local), through the multicast address of the destination.
template <int U>
__device__ void mc_store_piece(char* mc_dst, const char* src, long long nvec) {
  const long long stride = (long long)blockDim.x * U;
  for (long long v0 = threadIdx.x; v0 < nvec; v0 += stride) {
    uint4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      long long v = v0 + (long long)u * blockDim.x;
      if (v < nvec) r[u] = ld_vec(src + v * 16);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      long long v = v0 + (long long)u * blockDim.x;
      if (v < nvec) mc_st(mc_dst + v * 16, r[u]);
    }
  }
}

__device__ void record_failure(const InterpArgs& a, int code, int block, int lane, int wait);

// Books `need` ns on the link clock at *clock, starting no earlier than `ready`; returns the booking's end.  A
// compare-and-swap loop (bounded: after 4096 lost races the step is booked without the clock).
__device__ __forceinline__ unsigned long long pace_book(unsigned long long* clock, unsigned long long ready,
                                                        unsigned long long need) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(clock);
  for (int tries = 0; tries < 4096; ++tries) {
    const unsigned long long start = cur > ready ? cur : ready;
    const unsigned long long prev = atomicCAS(clock, cur, start + need);
    if (prev == cur) return start + need;
    cur = prev;
  }
  return ready + need;
}

// Staging state of one CTA: the mbarriers, the shared buffers and the running count of staged tiles (the same
// in every thread; a tile's buffer is count % kBulkStages and its mbarrier phase parity (count / kBulkStages) & 1).
struct BulkState {
  unsigned char* buf;
  uint32_t bar0;        // shared address of the first mbarrier (8 bytes apart)
  unsigned int issued;  // tiles whose loads thread 0 has issued
  unsigned int used;    // tiles consumed
};

// Waits (every thread) for tile `t`'s loads; false when the wait ran out of time or the launch is stopping.
__device__ bool bulk_wait(const InterpArgs& a, BulkState& bs, unsigned int t) {
  const uint32_t bar = bs.bar0 + 8u * (t % kBulkStages);
  const uint32_t parity = (t / kBulkStages) & 1u;
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  unsigned int spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0) {
      if (ld_volatile_int(&a.control->status) != ST_OK || ld_volatile_int(&a.control->abort_request)) return false;
      if (globaltimer() - t0 > a.timeout_ns) return false;
    }
  }
  return true;
}

// After a failure: wait (bounded) for every tile whose loads are still in flight, so nothing lands in
// shared memory after the CTA has moved on.
__device__ void bulk_drain(const InterpArgs& a, BulkState& bs) {
  for (unsigned int t = bs.used; t < bs.issued; ++t) {
    const uint32_t bar = bs.bar0 + 8u * (t % kBulkStages);
    const uint32_t parity = (t / kBulkStages) & 1u;
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity))
      if (globaltimer() - t0 > a.timeout_ns) break;
  }
  bs.used = bs.issued;
}

// dst[v] = scale? * op(src0[v], ..., src{K-1}[v]) over `bytes` bytes (a multiple of 16), the sources staged in
// shared memory by TMA bulk copies, kBulkStages - 1 tiles ahead of the tile being combined.  Thread 0 issues
// the copies; all threads combine and store.  A plain copy into this GPU's memory (`tma_store`: one source, no
// scale, local destination) leaves the store to TMA as well: thread 0 writes each staged tile back with a bulk
// store, and waits for those stores to have read a buffer before it refills it and for all of them to have
// completed before it returns.  Returns false (after draining) when a wait failed.
template <int DT, int RED>
__device__ bool move_bulk(char* dst, const char* const* src, int nsrc, long long bytes, bool do_scale, float scale,
                          const InterpArgs& a, BulkState& bs, bool tma_store) {
  using V = VecT<DT>;
  // bytes of one source per tile: the stage split evenly over the sources, in 1 KiB units
  const long long tile = (long long)((kBulkStageBytes / nsrc) & ~1023);
  const unsigned int tiles = (unsigned int)((bytes + tile - 1) / tile);
  const unsigned int first = bs.issued;   // tile numbers of this call: first .. first + tiles - 1
  auto issue = [&](unsigned int i) {      // thread 0 only
    const unsigned int t = first + i;
    const long long off = (long long)i * tile;
    const uint32_t n = (uint32_t)(bytes - off < tile ? bytes - off : tile);
    const uint32_t bar = bs.bar0 + 8u * (t % kBulkStages);
    unsigned char* stage = bs.buf + (size_t)(t % kBulkStages) * kBulkStageBytes;
    // the buffer was last read by a bulk store (copy mode) or through the generic proxy; either way those
    // reads come before the async-proxy writes that refill it
    if (tma_store) bulk_store_wait_read();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, n * (uint32_t)nsrc);
    for (int k = 0; k < nsrc; ++k) bulk_load(smem_addr(stage + (size_t)k * tile), src[k] + off, n, bar);
  };
  if (threadIdx.x == 0)
    for (unsigned int i = 0; i < tiles && i < (unsigned int)(kBulkStages - 1); ++i) issue(i);
  bs.issued += tiles < (unsigned int)(kBulkStages - 1) ? tiles : (unsigned int)(kBulkStages - 1);
  for (unsigned int i = 0; i < tiles; ++i) {
    const unsigned int t = first + i;
    if (i + kBulkStages - 1 < tiles) {
      if (threadIdx.x == 0) issue(i + kBulkStages - 1);
      ++bs.issued;
    }
    if (!__syncthreads_and(bulk_wait(a, bs, t))) {   // one decision for the whole CTA
      // a wait ran out of time: record it, let the loads in flight land, stop
      if (threadIdx.x == 0 && ld_volatile_int(&a.control->status) == ST_OK) record_failure(a, ST_TIMEOUT, -1, -1, -2);
      if (tma_store && threadIdx.x == 0) bulk_store_wait_all();
      bs.used = t;
      bulk_drain(a, bs);
      return false;
    }
    const unsigned char* stage = bs.buf + (size_t)(t % kBulkStages) * kBulkStageBytes;
    const long long off = (long long)i * tile;
    const long long n = bytes - off < tile ? bytes - off : tile;
    char* out = dst + off;
    if (tma_store) {
      if (threadIdx.x == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bulk_store(out, smem_addr(stage), (uint32_t)n);
      }
      bs.used = t + 1;
      continue;   // no thread touches the buffer; thread 0 alone orders its reuse
    }
    for (long long v = threadIdx.x; v < n / 16; v += blockDim.x) {
      uint4 r0 = *reinterpret_cast<const uint4*>(stage + v * 16);
      if (nsrc == 1 && !do_scale) {
        st_vec(out + v * 16, r0);
        continue;
      }
      float acc[V::N], tmp[V::N];
      V::unpack(r0, acc);
      for (int k = 1; k < nsrc; ++k) {
        V::unpack(*reinterpret_cast<const uint4*>(stage + (size_t)k * tile + v * 16), tmp);
#pragma unroll
        for (int e = 0; e < V::N; ++e) acc[e] = combine<RED>(acc[e], tmp[e]);
      }
      if (do_scale) {
#pragma unroll
        for (int e = 0; e < V::N; ++e) acc[e] *= scale;
      }
      st_vec(out + v * 16, V::pack(acc));
    }
    bs.used = t + 1;
    __syncthreads();   // every thread is done with this buffer before it is refilled
  }
  if (tma_store && threadIdx.x == 0) bulk_store_wait_all();
  return true;
}

// LEAN selects the register-lean unrolls (2 and 3 sources one vector deep, copies eight deep) that build
// without spills; PF adds the 256-byte L2 prefetch hint to the loads.
template <int DT, int RED, bool LEAN, bool PF = false>
__device__ void move_piece(char* dst, const char* const* src, int nsrc, long long nvec, bool do_scale, float scale) {
  switch (nsrc) {
    case 1: move_fixed<DT, RED, 1, LEAN ? 8 : 4, PF>(dst, src, nvec, do_scale, scale); break;
    case 2: move_fixed<DT, RED, 2, LEAN ? 1 : 2, PF>(dst, src, nvec, do_scale, scale); break;
    case 3: move_fixed<DT, RED, 3, LEAN ? 1 : 2, PF>(dst, src, nvec, do_scale, scale); break;
    case 4: move_fixed<DT, RED, 4, 1, PF>(dst, src, nvec, do_scale, scale); break;
    case 5: move_fixed<DT, RED, 5, 1, PF>(dst, src, nvec, do_scale, scale); break;
    case 6: move_fixed<DT, RED, 6, 1, PF>(dst, src, nvec, do_scale, scale); break;
    case 7: move_fixed<DT, RED, 7, 1, PF>(dst, src, nvec, do_scale, scale); break;
    case 8: move_fixed<DT, RED, 8, 1, PF>(dst, src, nvec, do_scale, scale); break;
    default: move_generic<DT, RED>(dst, src, nsrc, nvec, do_scale, scale); break;
  }
}

__device__ __forceinline__ unsigned long long* flag_ptr(const InterpArgs& a, int rank, long long index) {
  return reinterpret_cast<unsigned long long*>(a.base[rank] + a.flag_off) + index;
}

__device__ void record_failure(const InterpArgs& a, int code, int block, int lane, int wait) {
  if (atomicCAS(&a.control->status, ST_OK, code) == ST_OK) {
    a.control->detail[0] = a.rank;
    a.control->detail[1] = block;
    a.control->detail[2] = lane;
    a.control->detail[3] = wait;
  }
  __threadfence();
}

// Warp 0 waits for `n` flag targets; returns false when the CTA must stop.
__device__ bool wait_events(const InterpArgs& a, const DevWait* w, int n, int it, unsigned long long base, int block,
                            int lane) {
  const int l = threadIdx.x & 31;
  bool ok = true;
  for (int i = l; i < n && ok; i += 32) {
    const DevWait dw = w[i];
    unsigned long long target;
    const unsigned long long* f;
    if (dw.block < 0) {
      // a peer's start flag holds for the whole launch: checking it in the first iteration suffices
      if (it > 0) continue;
      target = base + 1;
      f = flag_ptr(a, dw.rank, a.start_slot);
    } else {
      int wit = dw.iter_delta < 0 ? a.niters * a.nbatch - 1 : it;
      target = base + (unsigned long long)wit * (unsigned long long)dw.stride + (unsigned long long)dw.event;
      f = flag_ptr(a, dw.rank, (long long)dw.block * kMaxFlagLanes + lane);
    }
    if (ld_acquire_sys(f) >= target) continue;
    const unsigned long long t0 = globaltimer();
    unsigned int spins = 0;
    while (ld_acquire_sys(f) < target) {
      if ((++spins & 63u) == 0) {
        if (ld_volatile_int(&a.control->status) != ST_OK || ld_volatile_int(&a.control->abort_request)) {
          ok = false;
          break;
        }
        if (globaltimer() - t0 > a.timeout_ns) {
          record_failure(a, ST_TIMEOUT, block, lane, i);
          ok = false;
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

template <int DT, int RED, bool LEAN, bool BULK>
__device__ void run_cta(const InterpArgs& a, int block, int lane, unsigned long long base, int* s_stop,
                        char* const* s_rank_base, const long long* s_buf_off, BulkState& bs) {
  const DevBlock blk = a.blocks[block];
  const int esize = DT == DT_F32 ? 4 : 2;
  const unsigned long long stride = 2ull * (unsigned long long)blk.nsteps;
  unsigned long long* my_flag = flag_ptr(a, a.rank, (long long)block * kMaxFlagLanes + lane);
  __shared__ const char* s_src[16];
  bool mc_pending = false;   // multimem or remote (push) stores of this thread not yet fenced
  const int total_iters = a.niters * a.nbatch;
  for (int it = 0; it < total_iters; ++it) {
    const int batch = it / a.niters;
    const PieceRange pr = piece_range(a.chunk_elems, a.piece_elems, it - batch * a.niters, a.nlanes, lane);
    for (int s = 0; s < blk.nsteps; ++s) {
      const DevStep st = a.steps[blk.step_begin + s];
      unsigned long long t_reach = 0, t_ready = 0, t_step0 = 0;
      if (a.trace_buf && threadIdx.x == 0) t_reach = globaltimer();
      if (st.wait_count) {
        if (threadIdx.x < 32) {
          bool ok = wait_events(a, a.waits + st.wait_begin, st.wait_count, it, base, block, lane);
          if (threadIdx.x == 0 && !ok) *s_stop = 1;
        }
        __syncthreads();
        if (*s_stop) return;
      }
      if (a.trace_buf && threadIdx.x == 0) t_ready = globaltimer();
      // link emulation times the transfer from here: waiting for the inputs does not use the emulated link
      if (a.pace_group > 0 && threadIdx.x == 0) t_step0 = globaltimer();
      const unsigned long long ev = base + (unsigned long long)it * stride + 2ull * s;
      if (st.flags & F_PUB_ARRIVE) {
        if (mc_pending) {
          asm volatile("fence.acq_rel.sys;" ::: "memory");
          mc_pending = false;
          __syncthreads();
        }
        if (threadIdx.x == 0) st_release_sys(my_flag, ev + 1);
      }
      if (st.op == OP_MC_ALLREDUCE && pr.hi > pr.lo) {
        const long long nvec = (pr.hi - pr.lo) * esize / 16;
        const DevSrc sr = a.srcs[st.src_begin];
        for (int k = 0; k < st.cnt; ++k) {
          const char* src = a.mc_base + s_buf_off[sr.buf] + batch * a.batch_stride[sr.buf] +
                            ((long long)(sr.chunk + k) * a.chunk_elems + pr.lo) * esize;
          char* dst = a.mc_base + s_buf_off[st.dst_buf] + batch * a.batch_stride[st.dst_buf] +
                      ((long long)(st.dst_chunk + k) * a.chunk_elems + pr.lo) * esize;
          mc_allreduce_piece<DT, LEAN ? 4 : 8>(dst, src, nvec, (st.flags & F_SCALE) != 0, a.scale);
        }
        mc_pending = true;
        if (s + 1 < blk.nsteps && a.steps[blk.step_begin + s + 1].op != OP_NOP) {
          // the next step may read what these multicast stores wrote: fence and join the CTA first
          asm volatile("fence.acq_rel.sys;" ::: "memory");
          mc_pending = false;
          __syncthreads();
        }
      }
      if (st.op == OP_MC_STORE && pr.hi > pr.lo) {
        const long long nvec = (pr.hi - pr.lo) * esize / 16;
        const DevSrc sr = a.srcs[st.src_begin];
        for (int k = 0; k < st.cnt; ++k) {
          const char* src = s_rank_base[a.rank] + s_buf_off[sr.buf] + batch * a.batch_stride[sr.buf] +
                            ((long long)(sr.chunk + k) * a.chunk_elems + pr.lo) * esize;
          char* dst = a.mc_base + s_buf_off[st.dst_buf] + batch * a.batch_stride[st.dst_buf] +
                      ((long long)(st.dst_chunk + k) * a.chunk_elems + pr.lo) * esize;
          mc_store_piece<LEAN ? 4 : 8>(dst, src, nvec);
        }
        mc_pending = true;
        if (s + 1 < blk.nsteps && a.steps[blk.step_begin + s + 1].op != OP_NOP) {
          // the next step may read what these multicast stores wrote: fence and join the CTA first
          asm volatile("fence.acq_rel.sys;" ::: "memory");
          mc_pending = false;
          __syncthreads();
        }
      }
      if ((st.op == OP_COPY || st.op == OP_REDUCE) && pr.hi > pr.lo) {
        const long long nvec = (pr.hi - pr.lo) * esize / 16;
        for (int k = 0; k < st.cnt; ++k) {
          if (threadIdx.x < st.nsrc && threadIdx.x < 16) {
            const DevSrc sr = a.srcs[st.src_begin + threadIdx.x];
            s_src[threadIdx.x] = s_rank_base[sr.rank] + s_buf_off[sr.buf] + batch * a.batch_stride[sr.buf] +
                                 ((long long)(sr.chunk + k) * a.chunk_elems + pr.lo) * esize;
          }
          __syncthreads();
          // a push writes the receiver's buffer through its peer mapping
          const int dr = (st.dst_rank >= 0 && st.dst_rank < a.nranks) ? st.dst_rank : a.rank;
          char* dst = s_rank_base[dr] + s_buf_off[st.dst_buf] + batch * a.batch_stride[st.dst_buf] +
                      ((long long)(st.dst_chunk + k) * a.chunk_elems + pr.lo) * esize;
          if (BULK && nvec * 16 >= kBulkMinBytes && st.nsrc <= 16) {
            const bool scaled = (st.flags & F_SCALE) != 0;
            const bool tma_store = (a.bulk & 2) != 0 && st.nsrc == 1 && !scaled && dr == a.rank;
            if (!move_bulk<DT, RED>(dst, s_src, st.nsrc, nvec * 16, scaled, a.scale, a, bs, tma_store)) {
              if (threadIdx.x == 0) *s_stop = 1;
              __syncthreads();
              return;
            }
          } else {
            // the register-lean instance (one rank by default) adds the L2 prefetch hint to its loads
            move_piece<DT, RED, LEAN, LEAN && !BULK>(dst, s_src, st.nsrc, nvec, (st.flags & F_SCALE) != 0, a.scale);
          }
          if (dr != a.rank) mc_pending = true;   // remote stores: fenced at system scope before the done flag
          __syncthreads();
        }
      }
      if (a.pace_group > 0 && (st.op == OP_COPY || st.op == OP_REDUCE) && threadIdx.x == 0 && pr.hi > pr.lo) {
        // link emulation: a step that pulled from another rank group books its bytes on this rank's emulated
        // link (one clock shared by all CTAs of the rank: a token bucket at the rank's share of the link) and
        // ends no earlier than its booking
        bool crosses = false;
        for (int i = 0; i < st.nsrc; ++i)
          crosses |= (a.srcs[st.src_begin + i].rank / a.pace_group) != (a.rank / a.pace_group);
        if (crosses) {
          const unsigned long long need =
              (unsigned long long)((double)(pr.hi - pr.lo) * esize * st.cnt * a.pace_ns_per_byte);
          const unsigned long long end = pace_book(&a.control->pace_clock, t_step0, need);
          // the wait is bounded by the booking itself, and by the launch timeout as a last resort
          const unsigned long long t0 = globaltimer();
          while (globaltimer() < end && globaltimer() - t0 < a.timeout_ns) {
          }
        }
      }
      if (st.flags & F_PUB_DONE) {
        if (mc_pending) {
          asm volatile("fence.acq_rel.sys;" ::: "memory");
          mc_pending = false;
        }
        __syncthreads();
        if (threadIdx.x == 0) st_release_sys(my_flag, ev + 2);
      }
      if (a.trace_buf && threadIdx.x == 0) {
        const long long slot = ((long long)blockIdx.x * a.trace_stride + (long long)it * blk.nsteps + s) * 3;
        if ((long long)it * blk.nsteps + s < a.trace_stride) {
          a.trace_buf[slot] = t_ready;
          a.trace_buf[slot + 1] = globaltimer();
          a.trace_buf[slot + 2] = t_ready - t_reach;
        }
      }
    }
  }
  // final event of this block: implies every event of every iteration
  if (mc_pending) asm volatile("fence.acq_rel.sys;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0)
    st_release_sys(my_flag, base + (unsigned long long)(total_iters - 1) * stride + 2ull * blk.nsteps);
  if (blk.end_wait_count) {
    if (threadIdx.x < 32) {
      bool ok = wait_events(a, a.waits + blk.end_wait_begin, blk.end_wait_count, total_iters - 1, base, block, lane);
      if (threadIdx.x == 0 && !ok) *s_stop = 1;
    }
    __syncthreads();
  }
}

// TL: record the launch timeline; LEAN: register-lean unrolls (see move_piece); BULK: copy and reduce steps
// stage their sources in shared memory with TMA bulk copies (move_bulk), kBulkSmemBytes of dynamic shared memory.
template <int DT, int RED, bool TL = false, bool LEAN = false, bool BULK = false>
__global__ void __launch_bounds__(512, 1) interp_kernel(const InterpArgs a) {
  __shared__ unsigned long long s_base;
  __shared__ int s_stop;
  __shared__ char* s_rank_base[kMaxRanks];
  __shared__ long long s_buf_off[BUF_COUNT];
  extern __shared__ __align__(1024) unsigned char s_dyn[];   // kBulkSmemBytes when a.bulk, else empty
  if (threadIdx.x < kMaxRanks) s_rank_base[threadIdx.x] = a.base[threadIdx.x];
  if (threadIdx.x < BUF_COUNT) s_buf_off[threadIdx.x] = a.buf_off[threadIdx.x];
  BulkState bs{s_dyn, smem_addr(s_dyn + (size_t)kBulkStages * kBulkStageBytes), 0u, 0u};
  if (BULK && threadIdx.x == 0) {
    for (int i = 0; i < kBulkStages; ++i) mbar_init(bs.bar0 + 8u * i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const int block = blockIdx.x / a.nlanes;
  const int lane = blockIdx.x % a.nlanes;
  if (threadIdx.x == 0) {
    s_base = (*(volatile unsigned long long*)&a.control->epoch) << 32;
    s_stop = 0;
    if (TL && blockIdx.x == 0) a.timeline[((s_base >> 32) % kTimelineSlots) * 2] = globaltimer();
    st_release_sys(flag_ptr(a, a.rank, a.start_slot), s_base + 1);
  }
  __syncthreads();
  // staged instances keep the lean unrolls for the pieces below kBulkMinBytes (fewer registers beside move_bulk)
  if (block < a.nblocks)
    run_cta<DT, RED, LEAN || BULK, BULK>(a, block, lane, s_base, &s_stop, s_rank_base, s_buf_off, bs);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int done = atomicAdd(&a.control->arrive, 1u);
    if (done == gridDim.x - 1) {
      if (TL) a.timeline[((s_base >> 32) % kTimelineSlots) * 2 + 1] = globaltimer();
      a.control->arrive = 0;
      a.control->epoch = a.control->epoch + 1;
      __threadfence();
    }
  }
}

// Cooperative launch of one interpreter instance; with TMA staging the instance gets its dynamic shared memory.
cudaError_t coop(const void* fn, dim3 grid, dim3 block, void** args, bool bulk, cudaStream_t stream) {
  size_t smem = 0;
  if (bulk) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmemBytes);
    if (e != cudaSuccess) return e;
    smem = kBulkSmemBytes;
  }
  return cudaLaunchCooperativeKernel(fn, grid, block, args, smem, stream);
}

template <int DT>
cudaError_t launch_red(const InterpArgs& a, cudaStream_t stream, int threads) {
  void* args[] = {const_cast<InterpArgs*>(&a)};
  dim3 grid(a.nblocks * a.nlanes), block(threads);
  const bool b = a.bulk != 0;
  if (b) {
    // the staged instances: every reduction, no timeline, the lean unrolls do not apply
    if (a.timeline) return cudaErrorInvalidValue;
    switch (a.redop) {
      case RED_PROD: return coop((void*)interp_kernel<DT, RED_PROD, false, false, true>, grid, block, args, b, stream);
      case RED_MIN: return coop((void*)interp_kernel<DT, RED_MIN, false, false, true>, grid, block, args, b, stream);
      case RED_MAX: return coop((void*)interp_kernel<DT, RED_MAX, false, false, true>, grid, block, args, b, stream);
      default: return coop((void*)interp_kernel<DT, RED_SUM, false, false, true>, grid, block, args, b, stream);
    }
  }
  if (a.timeline || a.lean) {
    // the instrumented and the lean instances exist for sum (and average) reductions and copies only
    if (a.redop != RED_SUM) return cudaErrorInvalidValue;
    if (a.timeline && a.lean)
      return coop((void*)interp_kernel<DT, RED_SUM, true, true>, grid, block, args, b, stream);
    if (a.timeline)
      return coop((void*)interp_kernel<DT, RED_SUM, true, false>, grid, block, args, b, stream);
    return coop((void*)interp_kernel<DT, RED_SUM, false, true>, grid, block, args, b, stream);
  }
  switch (a.redop) {
    case RED_PROD: return coop((void*)interp_kernel<DT, RED_PROD>, grid, block, args, b, stream);
    case RED_MIN: return coop((void*)interp_kernel<DT, RED_MIN>, grid, block, args, b, stream);
    case RED_MAX: return coop((void*)interp_kernel<DT, RED_MAX>, grid, block, args, b, stream);
    default: return coop((void*)interp_kernel<DT, RED_SUM>, grid, block, args, b, stream);
  }
}

}  // namespace

cudaError_t launch_interp(const InterpArgs& a, cudaStream_t stream, int threads) {
  if (a.nblocks < 1 || a.nlanes < 1 || a.niters < 1 || a.nbatch < 1 || threads < 32 || threads > 512 || threads % 32)
    return cudaErrorInvalidValue;
  if ((long long)a.niters * a.nbatch * 2ll * 65536ll >= (1ll << 32)) return cudaErrorInvalidValue;
  switch (a.dtype) {
    case DT_F32: return launch_red<DT_F32>(a, stream, threads);
    case DT_BF16: return launch_red<DT_BF16>(a, stream, threads);
    case DT_F16: return launch_red<DT_F16>(a, stream, threads);
    default: return cudaErrorInvalidValue;
  }
}

void apply_emulation_env(InterpArgs* a) {
  // VERICCL_EMULATE="group=4,gbps=25": pace data steps that read another group of 4 ranks as if each
  // group's inter-group traffic shared one 25 GB/s link: every rank of the group gets an even share
  // (25/4 GB/s), which its CTAs share through the rank's link clock (Control::pace_clock).
  const char* env = getenv("VERICCL_EMULATE");
  a->pace_group = 0;
  a->pace_ns_per_byte = 0.f;
  if (!env || !*env) return;
  int group = 0;
  double gbps = 0;
  if (sscanf(env, "group=%d,gbps=%lf", &group, &gbps) == 2 && group > 0 && gbps > 0) {
    a->pace_group = group;
    a->pace_ns_per_byte = (float)((double)group / gbps);
  }
}

int interp_max_ctas(int threads) {
  static int cached_threads[64] = {};
  static int cached_value[64] = {};
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cached_threads[dev] == threads && cached_value[dev] > 0) return cached_value[dev];
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // the smallest residency over the instances a launch may pick (dtype, timeline, lean), so a cooperative
  // grid sized from it is resident whichever instance runs
  // sized for the staged (TMA) launches too, which add kBulkSmemBytes of dynamic shared memory
  cudaFuncSetAttribute((const void*)interp_kernel<DT_BF16, RED_SUM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       kBulkSmemBytes);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, interp_kernel<DT_BF16, RED_SUM>, threads, kBulkSmemBytes);
  const void* others[] = {
      (const void*)interp_kernel<DT_F32, RED_SUM>, (const void*)interp_kernel<DT_BF16, RED_SUM, true, false>,
      (const void*)interp_kernel<DT_BF16, RED_SUM, false, true>, (const void*)interp_kernel<DT_F32, RED_SUM, false, true>,
      (const void*)interp_kernel<DT_BF16, RED_SUM, true, true>, (const void*)interp_kernel<DT_BF16, RED_SUM, false, false, true>,
      (const void*)interp_kernel<DT_F32, RED_SUM, false, false, true>};
  for (const void* fn : others) {
    int n = 0;
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmemBytes);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, kBulkSmemBytes) == cudaSuccess && n < per_sm)
      per_sm = n;
  }
  if (dev >= 0 && dev < 64) {
    cached_threads[dev] = threads;
    cached_value[dev] = sms * per_sm;
  }
  return sms * per_sm;
}

}  // namespace vb

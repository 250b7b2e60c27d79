// Device program: the compiled, per-rank form of an MSCCL-style XML schedule.
//
// The schedule's thread blocks become CTA groups ("blocks"); every block runs
// on `nlanes` CTAs, and each lane owns a fixed sub-range (a "piece") of every
// chunk, so the whole program is instantiated nlanes x niters times over
// disjoint element ranges.  Steps are pull-based (a receive loads the
// sender's source region directly from the sender's peer-mapped memory) or,
// in push mode, a send stores into the receiver's peer-mapped buffer.
// Cross-CTA and cross-rank ordering uses monotone 64-bit flags, one per
// (block, lane) per rank: step s of iteration it publishes
//   base + it * stride + 2*s + 1   when it arrives (its waits are satisfied)
//   base + it * stride + 2*s + 2   when it is done
// where base = epoch << 32 and stride = 2 * nsteps of the publishing block.
// These structs are plain data shared by the host compiler, the CPU
// interpreter and the CUDA kernel.
#pragma once
#include <stdint.h>

namespace vb {

enum BufId : uint8_t { BUF_IN = 0, BUF_OUT = 1, BUF_SCR = 2, BUF_COUNT = 3 };

enum OpKind : uint8_t {
  OP_NOP = 0,        // dependency / publication only
  OP_COPY = 1,       // dst = src0
  OP_REDUCE = 2,     // dst = op(src0, src1, ..., srcK-1)
  OP_MC_REDUCE = 3,  // dst(local) = op over the multicast group of src0 (multimem.ld_reduce)
  OP_MC_STORE = 4,   // multicast dst on every group member = src0 (multimem.st)
  OP_MC_ALLREDUCE = 5  // multicast dst = multimem.ld_reduce(src0): reduce + broadcast in one pass
};

enum StepFlags : uint16_t {
  F_SCALE = 1,        // multiply the result by the launch scale before storing
  F_PUB_ARRIVE = 2,   // publish the arrive event before the data operation
  F_PUB_DONE = 4,     // publish the done event after the data operation
};

enum DType : int32_t { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };
enum RedOp : int32_t { RED_SUM = 0, RED_PROD = 1, RED_MIN = 2, RED_MAX = 3 };

struct DevSrc {
  int16_t rank;   // owning rank (may be the local rank)
  uint8_t buf;    // BufId
  uint8_t pad;
  int32_t chunk;  // chunk offset inside the buffer
};

struct DevStep {
  uint8_t op;
  uint8_t dst_buf;
  uint16_t flags;
  int32_t dst_chunk;
  int32_t cnt;          // consecutive chunks
  int32_t src_begin;    // index into the source table
  int32_t nsrc;
  int32_t wait_begin;   // index into the wait table
  int32_t wait_count;
  int32_t dst_rank;     // rank whose buffer the step writes: < 0 (or the own rank) local; else a push into a peer
};

struct DevWait {
  int16_t rank;
  int16_t block;
  int32_t stride;       // stride (2*nsteps) of the target block
  int32_t event;        // event number inside one iteration (1-based)
  int32_t iter_delta;   // 0: same iteration; -1: the last iteration (end-of-kernel acknowledgements)
};

struct DevBlock {
  int32_t step_begin;
  int32_t nsteps;
  int32_t xml_tb;       // originating XML thread block id (-1 for a synthetic block)
  int32_t end_wait_begin;
  int32_t end_wait_count;
};

constexpr int kMaxRanks = 16;
constexpr int kMaxFlagLanes = 256;   // flag table stride per block

// Element range of one piece: lane `lane` of iteration `it` inside a chunk of
// `chunk_elems` elements.  `piece_elems` is a multiple of the vector width.
struct PieceRange { int64_t lo, hi; };

#if defined(__CUDACC__)
__host__ __device__
#endif
inline PieceRange piece_range(int64_t chunk_elems, int64_t piece_elems, int it, int nlanes, int lane) {
  int64_t piece = (int64_t)it * nlanes + lane;
  int64_t lo = piece * piece_elems;
  int64_t hi = lo + piece_elems;
  if (lo > chunk_elems) lo = chunk_elems;
  if (hi > chunk_elems) hi = chunk_elems;
  return PieceRange{lo, hi};
}

}  // namespace vb

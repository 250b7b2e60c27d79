// CPU reference interpreter of compiled device programs.
//
// Every (rank, block, lane) is a virtual CTA.  Virtual CTAs are advanced one
// step at a time in a seeded random order; a step runs only when all of its
// waits are satisfied, exactly as on the GPU, and a pull reads the peer's
// buffer at the moment the step runs.  Element arithmetic mirrors the kernel:
// sources are widened to fp32, combined left to right, scaled once when the
// step carries F_SCALE, and rounded back to the storage type.  A push step
// writes the receiving rank's buffer at the moment it runs.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <sstream>

#include "vb/plan.h"

namespace vb {
namespace {

float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);   // quiet NaN
  uint32_t rounding = 0x7fffu + ((u >> 16) & 1u);                               // round to nearest even
  return (uint16_t)((u + rounding) >> 16);
}

float load(const unsigned char* p, int dtype, long long i) {
  if (dtype == DT_F32) { float f; std::memcpy(&f, p + 4 * i, 4); return f; }
  uint16_t h;
  std::memcpy(&h, p + 2 * i, 2);
  if (dtype == DT_BF16) return bf16_to_f32(h);
  // fp16 -> fp32 (IEEE half, exact)
  uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, man = h & 0x3ff;
  float v;
  if (exp == 0) v = std::ldexp((float)man, -24);
  else if (exp == 31) v = man ? NAN : INFINITY;
  else v = std::ldexp((float)(man | 0x400), (int)exp - 25);
  return sign ? -v : v;
}

void store(unsigned char* p, int dtype, long long i, float v) {
  if (dtype == DT_F32) { std::memcpy(p + 4 * i, &v, 4); return; }
  uint16_t h;
  if (dtype == DT_BF16) {
    h = f32_to_bf16(v);
  } else {
    // fp32 -> fp16 round to nearest even via scaling arithmetic
    float a = std::fabs(v);
    uint16_t sign = std::signbit(v) ? 0x8000 : 0;
    if (std::isnan(v)) h = 0x7e00;
    else if (a >= 65520.0f) h = sign | 0x7c00;
    else if (a < std::ldexp(1.0f, -14)) {
      long long m = std::llrint(std::ldexp(a, 24));
      h = sign | (uint16_t)m;
    } else {
      int e;
      std::frexp(a, &e);   // a = f * 2^e, f in [0.5, 1)
      long long m = std::llrint(std::ldexp(a, 11 - e));   // 11 significant bits
      if (m == 2048) { m = 1024; ++e; }
      int exp = e - 1 + 15;
      if (exp >= 31) h = sign | 0x7c00;
      else h = sign | (uint16_t)(exp << 10) | (uint16_t)(m & 0x3ff);
    }
  }
  std::memcpy(p + 2 * i, &h, 2);
}

float combine(float a, float b, int redop) {
  switch (redop) {
    case RED_PROD: return a * b;
    case RED_MIN: return a < b ? a : b;
    case RED_MAX: return a > b ? a : b;
    default: return a + b;
  }
}

struct VCta {
  int rank, block, lane;
  int it = 0, s = 0;
  bool started = false, in_end = false, finished = false;
};

}  // namespace

InterpResult cpu_interpret(const CompiledPlan& plan, HostBuffers& bufs, int dtype, int redop, float scale,
                           long long chunk_elems, long long piece_elems, unsigned seed, int launches) {
  InterpResult res;
  const int P = (int)plan.ranks.size();
  const int L = plan.options.nlanes, I = plan.options.niters;
  const int esize = dtype == DT_F32 ? 4 : 2;
  int maxb = plan.max_blocks();
  size_t start_slot = (size_t)maxb * kMaxFlagLanes;
  std::vector<std::vector<uint64_t>> flags(P, std::vector<uint64_t>(start_slot + 1, 0));
  std::mt19937 rng(seed);
  auto base_ptr = [&](int rank, int buf) -> unsigned char* {
    auto& v = buf == BUF_IN ? bufs.in[rank] : buf == BUF_OUT ? bufs.out[rank] : bufs.scr[rank];
    return v.data();
  };
  auto buf_elems = [&](int rank, int buf) -> long long {
    auto& v = buf == BUF_IN ? bufs.in[rank] : buf == BUF_OUT ? bufs.out[rank] : bufs.scr[rank];
    return (long long)v.size() / esize;
  };
  for (int launch = 0; launch < launches; ++launch) {
    uint64_t base = (uint64_t)(launch + 1) << 32;
    std::vector<VCta> ctas;
    for (int r = 0; r < P; ++r)
      for (int b = 0; b < (int)plan.ranks[r].blocks.size(); ++b)
        for (int l = 0; l < L; ++l) ctas.push_back(VCta{r, b, l});
    size_t remaining = ctas.size();
    while (remaining) {
      std::vector<size_t> order(ctas.size());
      for (size_t i = 0; i < order.size(); ++i) order[i] = i;
      std::shuffle(order.begin(), order.end(), rng);
      bool progressed = false;
      for (size_t idx : order) {
        VCta& c = ctas[idx];
        if (c.finished) continue;
        const RankProgram& rp = plan.ranks[c.rank];
        const DevBlock& blk = rp.blocks[c.block];
        auto wait_ok = [&](int begin, int count, int it) {
          for (int w = 0; w < count; ++w) {
            const DevWait& dw = rp.waits[begin + w];
            if (dw.block < 0) {
              if (it == 0 && flags[dw.rank][start_slot] < base + 1) return false;
              continue;
            }
            int wit = dw.iter_delta < 0 ? I - 1 : it;
            uint64_t target = base + (uint64_t)wit * dw.stride + dw.event;
            if (flags[dw.rank][(size_t)dw.block * kMaxFlagLanes + c.lane] < target) return false;
          }
          return true;
        };
        auto publish = [&](int event, int it) {
          uint64_t v = base + (uint64_t)it * 2 * blk.nsteps + event;
          uint64_t& f = flags[c.rank][(size_t)c.block * kMaxFlagLanes + c.lane];
          if (v > f) f = v;
        };
        if (!c.started) {
          c.started = true;
          uint64_t& sf = flags[c.rank][start_slot];
          if (sf < base + 1) sf = base + 1;
          progressed = true;
          ++res.events;
          continue;
        }
        if (!c.in_end) {
          if (c.it >= I || blk.nsteps == 0) {
            c.in_end = true;
            publish(2 * blk.nsteps, I - 1);   // final event of the block
            progressed = true;
            continue;
          }
          const DevStep& st = rp.steps[blk.step_begin + c.s];
          if (!wait_ok(st.wait_begin, st.wait_count, c.it)) continue;
          if (st.flags & F_PUB_ARRIVE) publish(2 * c.s + 1, c.it);
          if (st.op == OP_COPY || st.op == OP_REDUCE) {
            PieceRange pr = piece_range(chunk_elems, piece_elems, c.it, L, c.lane);
            const int dr = (st.dst_rank >= 0 && st.dst_rank < P) ? st.dst_rank : c.rank;   // push target
            for (int k = 0; k < st.cnt; ++k) {
              long long dst_off = (long long)(st.dst_chunk + k) * chunk_elems;
              if (dst_off + pr.hi > buf_elems(dr, st.dst_buf)) {
                res.error = "destination out of range";
                return res;
              }
              unsigned char* dst = base_ptr(dr, st.dst_buf);
              for (long long e = pr.lo; e < pr.hi; ++e) {
                float acc = 0.f;
                for (int si = 0; si < st.nsrc; ++si) {
                  const DevSrc& sr = rp.srcs[st.src_begin + si];
                  long long off = (long long)(sr.chunk + k) * chunk_elems + e;
                  if (off >= buf_elems(sr.rank, sr.buf)) {
                    res.error = "source out of range";
                    return res;
                  }
                  float v = load(base_ptr(sr.rank, sr.buf), dtype, off);
                  acc = si == 0 ? v : combine(acc, v, redop);
                }
                if (st.flags & F_SCALE) acc *= scale;
                store(dst, dtype, dst_off + e, acc);
              }
            }
          } else if (st.op == OP_MC_ALLREDUCE || st.op == OP_MC_STORE) {
            // NVLS emulation: the switch reads the source chunk of every rank (ld_reduce, sum) or this
            // rank's source (st) and writes the result to the destination chunk of every rank
            PieceRange pr = piece_range(chunk_elems, piece_elems, c.it, L, c.lane);
            const DevSrc& sr = rp.srcs[st.src_begin];
            for (int k = 0; k < st.cnt; ++k) {
              long long src_off = (long long)(sr.chunk + k) * chunk_elems;
              long long dst_off = (long long)(st.dst_chunk + k) * chunk_elems;
              for (int q = 0; q < P; ++q)
                if (dst_off + pr.hi > buf_elems(q, st.dst_buf) || src_off + pr.hi > buf_elems(q, sr.buf)) {
                  res.error = "multicast range out of bounds";
                  return res;
                }
              for (long long e = pr.lo; e < pr.hi; ++e) {
                float acc = 0.f;
                if (st.op == OP_MC_ALLREDUCE) {
                  for (int q = 0; q < P; ++q) acc += load(base_ptr(q, sr.buf), dtype, src_off + e);
                } else {
                  acc = load(base_ptr(c.rank, sr.buf), dtype, src_off + e);
                }
                if (st.flags & F_SCALE) acc *= scale;
                for (int q = 0; q < P; ++q) store(base_ptr(q, st.dst_buf), dtype, dst_off + e, acc);
              }
            }
          } else if (st.op != OP_NOP) {
            res.error = "this op needs the GPU";
            return res;
          }
          if (st.flags & F_PUB_DONE) publish(2 * c.s + 2, c.it);
          progressed = true;
          ++res.events;
          if (++c.s == blk.nsteps) { c.s = 0; ++c.it; }
          continue;
        }
        if (!wait_ok(blk.end_wait_begin, blk.end_wait_count, I - 1)) continue;
        c.finished = true;
        --remaining;
        progressed = true;
      }
      if (!progressed) {
        std::ostringstream m;
        m << "deadlock in launch " << launch << ":";
        int shown = 0;
        for (auto& c : ctas)
          if (!c.finished && shown++ < 6) m << " (r" << c.rank << " b" << c.block << " l" << c.lane << " it" << c.it << " s" << c.s << (c.in_end ? " end" : "") << ")";
        res.error = m.str();
        return res;
      }
    }
  }
  res.ok = true;
  return res;
}

}  // namespace vb

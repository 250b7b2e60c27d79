// Per-step trace files of the interpreter (host side).
//
// The kernel stores, per CTA, three 64-bit %globaltimer values for every
// (iteration, step) it ran: when the step's waits were satisfied, when its
// data work ended, and how long it waited.  CTA c (block c / nlanes) owns
// slots [c * stride, (c + 1) * stride) with stride = niters * max_steps, and
// its record for (iteration i, step s) sits at slot i * nsteps(block) + s.
// A trace file is a 40-byte header {magic "VBTR", version 1, rank, CTAs,
// max steps, pad, records, reserved} followed by 64-byte records {cta, block,
// lane, iteration, step, op, start, end, wait, 16 bytes reserved}, all little
// endian; vericcl_b200/online/trace.py reads the same layout.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace vb {

constexpr uint32_t kTraceMagic = 0x56425452u;   // "VBTR"

struct TraceLayout {
  int rank = 0;
  int nlanes = 1, niters = 1, max_steps = 0;
  std::vector<std::vector<int>> block_ops;   // opcode of every step, per block
};

// Number of 64-bit words of the device trace buffer for this layout.
size_t trace_words(const TraceLayout& layout);
// Decode the raw buffer and write the trace file; returns the number of records written.
size_t write_trace_file(const std::string& path, const TraceLayout& layout, const std::vector<uint64_t>& raw);

}  // namespace vb

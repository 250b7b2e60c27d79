// Trace file writer shared by the C API and the native driver (no CUDA needed).
#include "vb/trace_io.h"

#include <cstdio>
#include <cstring>
#include <stdexcept>

namespace vb {

namespace {

template <typename T>
void put(std::vector<unsigned char>& out, T v) {
  unsigned char b[sizeof(T)];
  std::memcpy(b, &v, sizeof(T));   // the supported hosts are little endian
  out.insert(out.end(), b, b + sizeof(T));
}

}  // namespace

size_t trace_words(const TraceLayout& l) {
  return (size_t)l.block_ops.size() * (size_t)l.nlanes * (size_t)l.niters * (size_t)l.max_steps * 3;
}

size_t write_trace_file(const std::string& path, const TraceLayout& l, const std::vector<uint64_t>& raw) {
  if (raw.size() < trace_words(l)) throw std::runtime_error("trace buffer smaller than its layout");
  const size_t per_cta = (size_t)l.niters * (size_t)l.max_steps;
  std::vector<unsigned char> body;
  size_t records = 0;
  const int ctas = (int)l.block_ops.size() * l.nlanes;
  for (int cta = 0; cta < ctas; ++cta) {
    const int block = cta / l.nlanes, lane = cta % l.nlanes;
    const std::vector<int>& ops = l.block_ops[block];
    const int nsteps = (int)ops.size();
    for (int it = 0; it < l.niters; ++it)
      for (int s = 0; s < nsteps; ++s) {
        const size_t slot = (size_t)cta * per_cta + (size_t)it * nsteps + s;
        const uint64_t start = raw[slot * 3], end = raw[slot * 3 + 1], wait = raw[slot * 3 + 2];
        if (start == 0 && end == 0) continue;
        put<int32_t>(body, cta);
        put<int32_t>(body, block);
        put<int32_t>(body, lane);
        put<int32_t>(body, it);
        put<int32_t>(body, s);
        put<int32_t>(body, ops[s]);
        put<int64_t>(body, (int64_t)start);
        put<int64_t>(body, (int64_t)end);
        put<int64_t>(body, (int64_t)wait);
        body.insert(body.end(), 16, 0);
        ++records;
      }
  }
  std::vector<unsigned char> head;
  put<uint32_t>(head, kTraceMagic);
  put<uint32_t>(head, 1);
  put<int32_t>(head, l.rank);
  put<int32_t>(head, ctas);
  put<int32_t>(head, l.max_steps);
  put<int32_t>(head, 0);
  put<int64_t>(head, (int64_t)records);
  put<int64_t>(head, 0);
  const std::string tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot write trace file " + path);
  bool ok = std::fwrite(head.data(), 1, head.size(), f) == head.size() &&
            (body.empty() || std::fwrite(body.data(), 1, body.size(), f) == body.size());
  ok = (std::fclose(f) == 0) && ok;
  if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) throw std::runtime_error("cannot write trace file " + path);
  return records;
}

}  // namespace vb

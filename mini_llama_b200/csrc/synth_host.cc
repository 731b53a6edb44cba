// synth_host.cc — host (CPU) side of the seeded synthetic weight generator.
//
// Builds libmlb_synth.so, a CPU-only library (no CUDA), so the CPU oracles and
// the reference arm can be fed exactly the bytes the GPU generator writes
// (synth.h holds the shared definition). Multi-threaded over rows.
#include <stdint.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "synth.h"

namespace {

template <class F>
void parallel_rows(long long rows, int threads, F f) {
  if (threads <= 1 || rows < 64) {
    f(0, rows);
    return;
  }
  threads = (int)std::min<long long>(threads, rows);
  std::vector<std::thread> ts;
  for (int t = 0; t < threads; ++t) {
    long long a = rows * t / threads, b = rows * (t + 1) / threads;
    ts.emplace_back([=] { f(a, b); });
  }
  for (auto& th : ts) th.join();
}

}  // namespace

extern "C" {

uint64_t mlbs_stream_key(uint64_t seed, uint64_t stream) {
  return mlb::synth::stream_key(seed, stream);
}

uint64_t mlbs_stream_id(int kind, int layer) {
  return (uint64_t)kind * (1ull << 20) + (uint64_t)(layer < 0 ? 0 : layer);
}

// GGUF blocks for rows [row0, row0 + rows) and blocks [blk0, blk0 + nblk) of a
// [*, full_cols] tensor; row i is written at out + i * pitch.
void mlbs_gguf(int qtype, uint64_t key, float scale, int raw, long long row0, long long rows,
               long long blk0, long long nblk, long long full_cols, uint8_t* out, size_t pitch,
               int threads) {
  const int bsz = mlb::synth::block_bytes(qtype);
  const long long nb_full = (full_cols + 31) / 32;
  parallel_rows(rows, threads, [&](long long a, long long b) {
    for (long long r = a; r < b; ++r)
      for (long long j = 0; j < nblk; ++j) {
        uint8_t* o = out + (size_t)r * pitch + (size_t)j * bsz;
        if (raw)
          mlb::synth::raw_block(qtype, key, (uint64_t)((row0 + r) * nb_full + blk0 + j), o);
        else
          mlb::synth::synth_block(qtype, key, scale, row0 + r, blk0 + j, full_cols, o);
      }
  });
}

// fp32 values gauss(key, (row0+r)*full_cols + col0+c) * scale, row-major [rows, cols].
void mlbs_f32(uint64_t key, float scale, long long row0, long long rows, long long col0,
              long long cols, long long full_cols, float* out, int threads) {
  parallel_rows(rows, threads, [&](long long a, long long b) {
    for (long long r = a; r < b; ++r)
      for (long long c = 0; c < cols; ++c)
        out[r * cols + c] = mlb::synth::fmul(
            mlb::synth::gauss(key, (uint64_t)((row0 + r) * full_cols + col0 + c)), scale);
  });
}

// Quantises one block of n <= 32 values with the shared quantisers.
void mlbs_quantize_block(int qtype, const float* x, int n, uint8_t* out) {
  if (qtype == 1) mlb::synth::quantize_q8_0(x, n, out);
  else if (qtype == 2) mlb::synth::quantize_q4_0(x, n, out);
  else mlb::synth::quantize_q4_1(x, n, out);
}

uint16_t mlbs_f32_to_fp16(float f) { return mlb::synth::float_to_half_ref(f); }

}  // extern "C"

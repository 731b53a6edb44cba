// attention.cuh — split-K flash-decode attention (host-side interface).
#pragma once

#include "common.cuh"

namespace mlb {

struct AttnLaunch {
  const float* q = nullptr;       // [H][D]
  const float* keys = nullptr;    // layer base of the cache: [max_seq][KV][D]
  const float* values = nullptr;
  const int* pos_dev = nullptr;   // device position, or null to use pos_host
  int pos_host = 0;
  int H = 0, KV = 0, D = 0;
  int nsplit = 1;
  float scale = 1.0f;
  int include_current_v = 0;
  float* ws = nullptr;            // attn_ws_floats(...)
  int* counters = nullptr;        // KV ints, zero between launches
  float* out = nullptr;           // [H][D]
  // Batched rows (grid.z): row r of q/out at r * H * D, its own workspace
  // (attn_ws_floats per row) and KV counters; positions row_pos[r] (device)
  // and sequence row_seq[r] (device; null: row r) whose layer base is
  // keys + row_seq[r] * seq_stride.
  int rows = 1;
  const int* row_pos = nullptr;
  const int* row_seq = nullptr;
  long long seq_stride = 0;
  // Batched rows only: keys/values hold bf16 elements (same element
  // indexing, two bytes each); the scores and sums stay fp32.
  int kv_bf16 = 0;
};

void attn_check(int H, int KV, int D);
// The decode step needs the tiled kernel (device-side position).
void attn_check_tiled(int H, int KV, int D);
bool attn_tiled_ok(int H, int KV, int D);
int attn_splits(int KV, int sms, int max_seq);
size_t attn_ws_floats(int H, int KV, int D, int nsplit);
size_t attn_smem_bytes(int G, int D);
void attn_launch(const AttnLaunch& l, cudaStream_t stream, bool pdl);

// 1/sqrt(D) evaluated like the reference CPU path (src/forward.cc:489): the
// quotient in double, stored as float.
float attn_scale(int head_dim);

}  // namespace mlb

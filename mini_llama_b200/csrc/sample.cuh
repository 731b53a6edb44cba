// sample.cuh — token sampling on the device: MiniSampler::Sample
// (src/sampler.cc:107-183) over a logits row already in device memory, with
// its Mersenne Twister state resident on the device, so a decode loop that
// samples needs no per-step logits download or host round trip.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace mlb {

constexpr int kMtN = 624;              // MT19937 state words
constexpr int kSampleMaxTopK = 4096;   // candidates a device top-k sample sorts

// std::mt19937's state, laid out for the device (one generator per sampler).
struct MtState {
  uint32_t mt[kMtN];
  int idx;  // next word to temper; kMtN = regenerate first
};

// State of std::mt19937 seeded with `seed` (the generator's standard seeding
// recurrence), on the host.
void mt_seed(uint32_t seed, MtState* out);

// One sample (the device form of MiniSampler::Sample, parameters already
// validated): logits [n] on the device; *out_id receives the id. When token
// is non-null the id also becomes the context's next input token and
// replaces tokens[*step - 1] (the step that produced the logits has already
// advanced step and written its greedy id there). A non-finite logit records
// MLB_ERR_INVALID at site 700 in *status and leaves the outputs untouched.
// Draws one 32-bit word from *st only when the reference would (temperature
// >= 1e-6 and top_k != 1).
void sample_launch(const float* logits, int n, float temperature, int top_k, MtState* st,
                   int* out_id, DeviceStatus* status, int* token, int* tokens, const int* step,
                   cudaStream_t stream);

}  // namespace mlb

// step.cuh — the persistent decode-step kernel (host-side interface).
//
// One cooperative launch computes a whole decode step of a single-GPU model:
// every quantised projection, attention, the lm_head with the greedy argmax,
// and the token/position update. The grid is one CTA per SM; ops are phases
// separated by grid barriers, and each warp's weight stream runs ahead across
// phase boundaries (see step.cu).
#pragma once

#include <vector>

#include "gemv.cuh"

namespace mlb {

enum StepPhaseKind : int { kPhaseGemv = 0, kPhaseAttn = 1 };

struct StepGemv {
  const uint8_t* w;     // super-block array
  int sbb;              // bytes per super-block
  int ntiles, nchunks, gc, ngroups;
  long long nsb;
  int k;
  const float* x;       // activation row; null = the embedding row of the step's token
  const float* norm_w;  // fused RMSNorm of x when non-null
  float eps;
  EpiParams epi;        // kEpiResidual with resid null: residual = the embedding row
  // Tensor parallel: tp_ar >= 0 marks a phase whose epilogue writes exchange
  // step tp_ar of this decode step into every rank as tagged words
  // (kEpiTpPartial, slot epi.tp_slot); before the barrier that ends the phase
  // each CTA adds its tiles of the exchange to epi.resid (null: the embedding
  // row) into epi.y, with per-tile sums of squares into epi.ss_out.
  int tp_ar;
  // RMSNorm statistic of x as the producing phase's per-tile sums of squares
  // (ss_n tiles), or null
  const float* ss_in;
  int ss_n;
};

struct StepAttn {
  const float* q;       // [H][D]
  const float* keys;    // layer base of the cache [max_seq][KV][D]
  const float* values;
  float* out;           // [H][D]
  int H, KV, D;
  float scale;
  int include_current_v;
  int kv_bf16;          // keys/values hold bf16 elements
};

struct alignas(16) StepPhase {  // copied into shared memory 16 bytes at a time
  int kind;
  StepGemv g;
  StepAttn at;
};

// One CTA's share of one GEMV phase, computed on the host (entry
// [phase][cta]; entries of attention phases are unused). The range is whole
// group-tiles; it splits into at most two segments, one per chunk group, each
// a run of whole tiles of that group.
struct alignas(16) StepCta {
  const uint8_t* w;  // its first super-block
  int cb, ce;        // super-block range [cb, ce)
  int next;          // the next GEMV phase (nphases: none)
  int nseg;          // segments (0 when the range is empty)
  int T[2];          // tiles of each segment
  int nc[2];         // chunks per tile in each segment (its group's width)
  int grp[2];        // chunk group of each segment
  int t0[2];         // first tile of each segment
  int pad[2];
};

struct StepArgs {
  const StepPhase* phases;  // device array
  const StepCta* cta;       // device array [nphases][grid]
  int nphases;
  int sb_stride;            // bytes per ring slot (largest super-block)
  int stages;               // ring slots per warp
  int scratch_bytes;        // per-phase shared scratch
  const float* embedding;
  int dim;
  int* token;               // device scalars of the context
  int* pos;
  int* step;
  int* tokens;
  unsigned long long* argmax_key;
  float* ws;                // GEMV fix-up partials
  int* counters;            // GEMV fix-up arrival counters (zero between phases)
  float* attn_ws;           // attention slice records [max(grid, KV)][gq][D + 4]
  int* attn_counters;       // [KV] (zero between phases)
  unsigned int* sync;       // [0] grid-barrier arrivals, [1] end-of-step arrivals
  DeviceStatus* status;
  // tensor parallel (null tp on one GPU): the exchange; tp_gen[0] counts the
  // exchange steps and tp_gen[1] the decode steps completed (same on every
  // rank); tp_steps exchange steps per decode step (two per layer)
  const TpXchg* tp;
  unsigned int* tp_gen;
  int tp_steps;
  // optional phase trace (null: none): global-timer nanoseconds per phase p
  // and CTA c at [(p * grid + c) * 2]: the start of the phase's work (after
  // the barrier ahead of it) and, at + 1, its end (before the next barrier)
  unsigned long long* trace;
};

// Launch plan of the step kernel for one context.
struct StepPlan {
  bool ok = false;
  std::string why;          // reason the step kernel is not used, when !ok
  int qtype = 0, gq = 0, grid = 0, stages = 0, sb_stride = 0, scratch_bytes = 0;
  size_t smem = 0;
  int nphases = 0;
  void* phases = nullptr;   // device StepPhase array (owned by the context)
  void* cta = nullptr;      // device StepCta array [nphases][grid] (owned by the context)
  size_t attn_ws_floats = 0;
};

// Shared memory the step kernel needs for a scratch size and ring shape.
size_t step_smem_bytes(int scratch_bytes, int sb_stride, int stages, int nphases);
// Scratch one GEMV phase needs (staged x, run slots, reduction space).
int step_gemv_scratch(const QMatrix& m);
// Scratch the attention phase needs.
int step_attn_scratch(int gq, int D);
// Whether a matrix can be a phase of the step kernel on `grid` CTAs (at most
// two chunk groups per CTA range); otherwise sets why.
bool step_gemv_ok(const QMatrix& m, int grid, std::string* why);
bool step_attn_ok(int H, int KV, int D, std::string* why);

// The per-CTA table of a phase list on `grid` CTAs.
std::vector<StepCta> step_cta_table(const std::vector<StepPhase>& ph, int grid);

// Makes one of the step kernel's bounded waits run out on the current device
// (which = 0: a ring mbarrier, 1: a grid barrier) with a limit of
// limit_cycles SM cycles; returns the recorded status code and site.
void step_wait_selftest(int which, long long limit_cycles, int where, int* code, int* at);

// Launches one step (cooperative launch, capturable in a CUDA graph).
void step_launch(const StepPlan& plan, const StepArgs& args, cudaStream_t stream);
// Resident blocks of the step kernel per SM with `smem` bytes of shared memory.
int step_max_blocks_per_sm(int qtype, int gq, size_t smem);

}  // namespace mlb

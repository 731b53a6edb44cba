// qgemm.cuh — quantised GEMM on the 5th-generation tensor cores (tcgen05),
// for batches of activation rows (batched decode and prompt prefill).
//
// y[r, n] = sum_k W[n, k] x[r, k] for M activation rows against a weight in
// the super-block layout of gemv.cuh (the same resident bytes the batch-1 path
// streams). Per CTA tile of 128 weight rows:
//   * a producer warp bulk-copies, per 256-input chunk, the 8 super-blocks of
//     the tile and the chunk of the staged activations into a shared-memory
//     ring (mbarrier complete_tx);
//   * 8 dequantising warps turn each code into its exact value w = d * q
//     (Q4_1: d * q + m) split as fp16 hi + lo (w - hi, exact for Q4_0 / Q8_0),
//     and store them into tensor memory (tcgen05.st) as the MMA's A operand,
//     one TMEM lane per weight row;
//   * one elected thread issues tcgen05.mma.kind::f16 with A from TMEM and B =
//     the activations staged as fp16 hi (columns [0, Mp)) and lo (columns
//     [Mp, 2 Mp)) in the canonical K-major layout: D += W_hi [x_hi | x_lo] and
//     D += W_lo x_hi into one fp32 accumulator in TMEM (the W_lo x_lo term is
//     below 2^-22 relative and dropped);
//   * the same 8 warps read D back (tcgen05.ld), add the hi and lo columns and
//     run the fused epilogue (store / residual / SwiGLU / QKV with per-row
//     RoPE position and KV-cache slot / greedy argmax per row).
// The (tile, chunk) units are split evenly over a persistent grid of one CTA
// per SM; a tile split over CTAs leaves fp32 partials in a workspace and the
// last CTA to finish it sums them in chunk order, so results do not depend on
// timing.
#pragma once

#include "gemv.cuh"

namespace mlb {

constexpr int kTcRows = 128;      // weight rows per CTA tile (MMA M)
constexpr int kTcMaxMp = 64;      // padded batch rows per pass (MMA N = 2 Mp <= 128)

// Activation rows padded for the MMA (N = Mp and 2 Mp must be multiples of 16).
inline int tc_mp(int rows) { return rows <= 16 ? 16 : (rows + 15) / 16 * 16; }
// Bytes of one 256-input chunk of staged activations: 2 Mp rows of 256 fp16
// inputs (hi rows, then lo rows), then 2 Mp rows of the 16 half-block sums of
// those inputs (the Q4_1 min term).
#if defined(__CUDACC__)
__host__ __device__
#endif
inline size_t tc_chunk_bytes(int mp) { return (size_t)mp * 1088; }

// Per-row epilogue of the batched GEMM: what happens to output row n of batch
// row r (r < rows).
struct BEpi {
  int kind;            // kEpiStore, kEpiResidual, kEpiSwiglu, kEpiQkv
  int rows;            // batch rows
  float* y;            // [rows][ldy]
  int ldy;
  int n_out;           // logical output rows
  const float* resid;  // kEpiResidual: [rows][ldr]
  int ldr;
  // kEpiQkv: per-row position and sequence; the layer base of sequence s's
  // cache is keys + s * seq_stride (rows [max_seq][kv_rows])
  int q_rows, kv_rows, k_off, v_off, head_dim, neox;
  const float* bias;
  const float2* rope;
  const int* row_pos;
  const int* row_seq;  // null: sequence = row
  float* keys;
  float* values;
  long long seq_stride;
  int kv_bf16;         // keys/values hold bf16 elements (rounded to nearest even)
  float* q_out;        // [rows][q_rows]
  // greedy argmax per batch row (kEpiStore): keys_out[r] folds
  // argmax_key_of(value, argmax_base + n) with atomicMax
  unsigned long long* argmax_keys;
  int argmax_base;
};

struct TcWorkspace {
  float* partials = nullptr;   // split-tile partials
  size_t partial_floats = 0;
  int* counters = nullptr;     // one per row tile, zero between launches
  int counter_count = 0;
  DeviceStatus* status = nullptr;
};

// Staged activations: x [rows][ldx] (optionally RMS-normalised with norm_w,
// row by row) -> fp16 hi/lo in the B layout of `chunks` 256-input chunks.
// Rows >= rows and inputs >= k stage as zero. gather (optional): row r of x is
// table + gather[r] * ldx (the embedding rows of the step's tokens).
// pdl: launch with programmatic dependent launch (the kernel waits for the
// previous one before reading its data).
void tc_stage_launch(const float* x, int ldx, int rows, int k, int chunks, const float* norm_w,
                     float eps, const int* gather, uint8_t* staged, cudaStream_t stream,
                     bool pdl = false);

// Scratch sizes for a matrix at `rows` activation rows on `grid` CTAs.
size_t tc_partial_floats(const QMatrix& m, int rows, int grid);
int tc_counter_count(const QMatrix& m);

// y = W x for the staged activations (rows <= kTcMaxMp), epilogue `epi`.
// grid_ctas 0 = one CTA per SM.
// pdl: programmatic dependent launch; the first stages' weight copies are
// issued before the kernel waits for the previous one.
void tc_gemm_launch(const QMatrix& m, const uint8_t* staged, int rows, const BEpi& epi,
                    const TcWorkspace& ws, cudaStream_t stream, int grid_ctas = 0,
                    bool pdl = false);

// Whether the tensor-core GEMM takes this matrix (quantised, k <= 2^20).
bool tc_gemm_ok(const QMatrix& m, int rows);

}  // namespace mlb

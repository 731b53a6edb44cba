// gemv.cuh — quantised GEMV for the decode path (host-side declarations).
//
// Layout ("super-block" layout). A weight [N, K] in GGUF blocks is repacked
// once into super-blocks (SB) of 16 output rows x 256 inputs (8 GGUF blocks):
//   Q4_0: 2048 B nibbles + 256 B fp16 scales            = 2304 B
//   Q4_1: 2048 B nibbles + 256 B scales + 256 B mins     = 2560 B
//   Q8_0: 4096 B int8    + 256 B scales                  = 4352 B
// The bytes inside an SB are ordered so that lane l of a warp reads exactly
// the mma.sync A-fragment data it needs with 16-byte loads (see gemv.cu).
// SBs are ordered (chunk-group, tile, chunk) so that a contiguous range of
// SBs is a contiguous range of memory; the GEMV gives each warp an equal
// contiguous range (stream-K) and finishes split tiles deterministically.
// Rows beyond N and inputs beyond K are zero blocks (scale 0). The bytes
// streamed per GEMV equal the GGUF bytes up to this padding.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace mlb {

constexpr int kTileRows = 16;
constexpr int kChunkK = 256;
constexpr int kGemvWarps = 16;  // warps per CTA, one CTA per SM
constexpr int kMaxBatch = 4;  // batch rows one pass of the MMA GEMV carries
constexpr int kMaxStages = 4;  // deepest per-warp weight ring (barrier slots)
// Ring depth used: two super-blocks per warp (74-139 KB in flight per SM).
// Measured on B200 with the ring alone, 2 slots x 16 warps of 2304 B stream
// at 7.2 TB/s and 4 slots at 5.9 TB/s: more bytes in flight only queue.
constexpr int kRingStages = 2;

inline int sb_bytes(int qtype) {
  return qtype == MLB_Q8_0 ? 4352 : (qtype == MLB_Q4_1 ? 2560 : 2304);
}
inline size_t gguf_row_bytes(int qtype, int k) {
  if (qtype == MLB_F32) return (size_t)k * 4;
  size_t nb = (size_t)(k + 31) / 32;
  return nb * (qtype == MLB_Q8_0 ? 34 : (qtype == MLB_Q4_1 ? 20 : 18));
}

// Epilogue selectors: what happens to each finished output row.
enum EpiKind : int {
  kEpiStore = 0,    // y[r, row] = v
  kEpiResidual = 1, // y[r, row] = resid[r, row] + v
  kEpiQkv = 2,      // + bias, RoPE, q -> q_out, k/v -> KV cache slot (layer, *pos)
  kEpiSwiglu = 3,   // tile rows 0..7 gate, 8..15 up -> y[r, 8t+i] = silu(g) * u
  kEpiTpPartial = 4,  // tensor parallel: v -> every rank's partial slot [tp_slot][me][row]
};

// Rank-to-rank exchange of one tensor-parallel context: each rank owns one
// exchange buffer, and every rank's buffer is mapped into every process
// (peers[r]; peers[me] is the local one). Byte offsets inside a buffer:
// partial sums [2 slots][n][dim] as tagged 8-byte words {fp32 bits, exchange
// step + 1} (an 8-byte store arrives whole, so the data is its own signal),
// full logits [vocab] fp32, argmax keys [n] u64 and key counters [n] u32
// (kflags[r]: rank r's greedy keys delivered, one per decode step).
constexpr int kMaxTp = 8;
struct TpXchg {
  int n, me, dim, vocab;
  long long parts_off, logits_off, keys_off, kflags_off;
  uint8_t* peers[kMaxTp];
};

struct EpiParams {
  int kind;
  float* y;
  int ldy;
  int n_out;           // valid output rows (logical)
  const float* resid;  // kEpiResidual
  int ldr;
  // kEpiQkv
  int q_rows, kv_rows;        // logical rows of the q and of the k (= v) sections
  int k_off, v_off;           // tile-aligned section offsets in the fused matrix
  int head_dim;
  int neox;                   // rows are stored pair-interleaved within heads
  const float* bias;          // fused [q | k | v] logical bias or null
  const float2* rope;         // [max_seq][head_dim/2] (cos, sin)
  const int* pos;             // device scalar
  float* keys;                // cache slot base of this layer: + pos * kv_rows
  float* values;
  int kv_bf16;                // the cache holds bf16 elements (rounded to nearest even)
  float* q_out;
  // Greedy argmax fused into a store epilogue (batch row 0): every finished
  // tile folds its rows into *argmax_key with atomicMax on
  // (order-preserving float bits << 32 | ~index); argmax_base offsets the index
  // (vocabulary shard start under tensor parallelism).
  unsigned long long* argmax_key;
  int argmax_base;
  // Tensor parallel (step kernel): kEpiTpPartial writes partial sums into
  // slot tp_slot of every rank; kEpiStore with tp set writes the logits rows
  // (global index argmax_base + row) into every rank's exchange buffer.
  const TpXchg* tp;
  int tp_slot;
  unsigned int tp_tag;  // kEpiTpPartial: tag of this exchange step (set on the device)
  // kEpiResidual, one batch row: ss_out[tile] = the sum of squares of the
  // tile's 16 output rows (fixed order), for the next phase's RMSNorm
  float* ss_out;
  // Step kernel (set on the device): resid_s, when set, holds the residual
  // rows of tiles resid_t0.. (batch row 0) in shared memory; pos_set marks
  // pos_now as the position (else *pos is read); rope_s, when set, holds the
  // position's rope row (head_dim / 2 float2) in shared memory
  const float* resid_s;
  int resid_t0;
  int pos_set, pos_now;
  const float2* rope_s;
};

#if defined(__CUDACC__)
// Key whose unsigned order is (value, then lower index) order; NaN maps to 0
// and never wins, as in ArgMax (src/ops.cc:226-231, `x > best` is false for NaN).
__device__ __forceinline__ unsigned long long argmax_key_of(float v, int index) {
  if (v != v) return 0ull;
  unsigned int u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)index);
}
__device__ __forceinline__ int argmax_index_of(unsigned long long key) {
  return key == 0ull ? 0 : (int)(0xFFFFFFFFu - (unsigned int)(key & 0xFFFFFFFFull));
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}
#endif

// Index of the super-block of tile t, chunk c in the (chunk group, tile,
// chunk) order.
#if defined(__CUDACC__)
__host__ __device__
#endif
inline long long sb_index(int t, int c, int ntiles, int nchunks, int gc) {
  const int grp = c / gc;
  const int cc = c - grp * gc;
  const int geff = gc < nchunks - grp * gc ? gc : nchunks - grp * gc;
  return (long long)grp * ntiles * gc + (long long)t * geff + cc;
}

struct QMatrix {
  int qtype = 0;
  int n = 0, k = 0;          // logical shape [n, k]
  int ntiles = 0, nchunks = 0;
  int gc = 0, ngroups = 0;   // chunks per group and group count
  long long nsb = 0;         // super-blocks
  size_t bytes = 0;          // device bytes (SB array or F32 rows)
  size_t gguf_bytes = 0;     // algorithmic GGUF bytes
  uint8_t* data = nullptr;   // device
  bool owns = true;
  mutable int grid_cache[3] = {0, 0, 0};  // launch grid per batch width (1, 2, 4)
};

// Geometry for a [n, k] weight of qtype with group size chosen for batch M.
void qmatrix_geometry(QMatrix& m, int qtype, int n, int k, int max_batch);
// Repacks GGUF blocks (device, [n, k] with row pitch gguf_row_bytes) into m.data.
// row_map (device, optional) gives the source row for each destination row
// (-1 = zero row); used to fuse / interleave / permute matrices.
void qmatrix_repack(const QMatrix& m, const uint8_t* src, size_t src_pitch,
                    const int* row_map, int col_block0, cudaStream_t stream);

struct GemvWorkspace {
  float* partials = nullptr;  // >= ntiles * nchunks * 16 * M floats
  size_t partial_floats = 0;
  int* counters = nullptr;    // >= ntiles ints, zero between launches
  size_t counter_count = 0;
  DeviceStatus* status = nullptr;
};

struct NormSpec {
  const float* weight = nullptr;  // fused RMSNorm on x when non-null
  float eps = 0.0f;
};

// y-rows of the matrix against x[rows, ldx] (rows <= kMaxBatch), fused
// norm/epilogue. grid_ctas 0 = one CTA per SM. pdl: launch with programmatic
// dependent launch.
void gemv_launch(const QMatrix& m, const float* x, int rows, int ldx, const NormSpec& norm,
                 const EpiParams& epi, const GemvWorkspace& ws, cudaStream_t stream, bool pdl,
                 int grid_ctas = 0);
// Number of kernels gemv_launch issues for `rows` (>= 1).
int gemv_kernel_count(const QMatrix& m, int rows);

// Dequantised fp32 [n, k] (row-major, device) of a quantised matrix, decoded
// from its super-block layout.
void qmatrix_dequant(const QMatrix& m, float* out, cudaStream_t stream);

// Generic GEMV straight over raw GGUF blocks (any shape; the standalone API).
void gemv_gguf(int qtype, const float* x, int rows, int k, const void* w, int n, float* y,
               cudaStream_t stream);

// Seeded synthetic fill of m (GGUF blocks generated on the device, then repacked).
void qmatrix_synthesize(const QMatrix& m, uint64_t key, float scale, int raw,
                        long long row0, long long full_rows, long long col0, long long full_cols,
                        const int* row_map, cudaStream_t stream);
// Fills GGUF blocks [rows, blocks] (device) of the seeded generator; rows are
// global rows row0.., blocks are global blocks blk0.. of a [*, full_cols] tensor.
void synth_gguf_blocks(int qtype, uint64_t key, float scale, int raw, long long row0,
                       long long rows, long long blk0, long long nblk, long long full_cols,
                       uint8_t* dst, size_t dst_pitch, cudaStream_t stream);
// fp32 tensor values gauss(key, index) * scale for rows row0.. and columns col0..
void synth_f32(uint64_t key, float scale, long long row0, long long rows, long long col0,
               long long cols, long long full_cols, float* dst, cudaStream_t stream);

}  // namespace mlb

// qgemm.cu — tcgen05 quantised GEMM for batches of activation rows.
//
// Reference: the reference runs a batch as one ForwardToken per token
// (ForwardBatch, src/batch.cc:35-50), so its linear layers are always
// matrix-vector products (LinearQ80/Q40/Q41, src/quant.cc:365-471, and the
// CUDA Q*LinearKernel, src/cuda_quant.cu:36-130). Here a batch of rows streams
// each weight once through the tensor cores. See qgemm.cuh for the data flow.
//
// Roles (10 warps, one CTA per SM):
//   warp 0      producer: bulk copies of super-blocks and staged activations
//   warp 1      TMEM allocation; lane 0 issues tcgen05.mma and commits
//   warps 2..9  dequantise into TMEM (A operand); epilogue from TMEM (D)
// Warp w may only touch TMEM lanes 32 (w % 4) .. 32 (w % 4) + 31, so the 8
// dequantising warps cover the four lane quadrants twice: warps 2..5 take the
// first two blocks of every 4-block half chunk, warps 6..9 the other two, and
// in the epilogue the first or second half of the batch columns. Each of the
// 8 (quadrant, column half) slices of a tile is finished by its own warp, so
// no CTA-wide barrier is needed after the main loop.
//
// Every wait is bounded: on a timeout the waiting thread records
// MLB_ERR_TIMEOUT in the status word and raises the CTA's abort flag; all
// roles leave their loops, outstanding bulk copies and MMAs are waited for
// (bounded), TMEM is released and the CTA exits.
#include "qgemm.cuh"

#include <cuda_bf16.h>

#include <algorithm>

namespace mlb {

namespace {

constexpr int kTcWarps = 10;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kDqWarps = 8;  // one arrival per dequantising warp on afull / dempty
constexpr int kTmemCols = 512;
constexpr int kAStageCols = 128;  // one 128-input half chunk: hi 64 columns + lo 64 columns
constexpr int kDCol = 256;        // accumulator columns [256, 256 + 2 Mp)
constexpr int kMinCol = 384;      // Q4_1 min-term A operand: 8 columns (16 fp16 mins)
constexpr int kMaxRingStages = 4;
constexpr long long kTcWaitCycles = 2000000000LL;  // about 1 s

// ------------------------------------------------------------ tcgen05 PTX

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// The mbarrier tracks the completion of every tcgen05 operation this thread
// issued before it.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem descriptor]; accumulate = 0 overwrites D.
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  const uint32_t z = 0u;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 8 consecutive columns of this thread's lane, then the wait for the load
// (the registers pass through the wait so nothing reads them earlier).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                 "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7])::"memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// Shared-memory matrix descriptor of a K-major, non-swizzled operand whose 8
// x 16-byte core matrices sit 128 bytes apart along K (leading byte offset)
// and `sbo` bytes apart along the rows (stride byte offset); version 1 (sm100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor, kind::f16: fp16 A and B, fp32 D, both K-major,
// M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// ------------------------------------------------------------ staging (B)

// Byte offset of (activation row n of 2 Mp, input k) in the staged buffer.
__device__ __forceinline__ size_t staged_off(int n, int k, size_t chunk_bytes) {
  const int c = k >> 8, kk = k & 255;
  return (size_t)c * chunk_bytes + (size_t)(n >> 3) * 4096 + (size_t)(kk >> 3) * 128 +
         (size_t)(n & 7) * 16 + (size_t)(kk & 7) * 2;
}

constexpr int kStageThreads = 128;
constexpr int kStageChunks = 4;  // chunks per CTA (128 threads x 8 inputs)

// Eight consecutive inputs from k0 of a row of length k (zeros past the end).
__device__ __forceinline__ void load8(const float* row, int k0, int k, float (&e)[8]) {
  if (k0 + 7 < k && ((((uintptr_t)(row + k0)) & 15) == 0)) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(row + k0));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(row + k0 + 4));
    e[0] = a.x; e[1] = a.y; e[2] = a.z; e[3] = a.w;
    e[4] = b.x; e[5] = b.y; e[6] = b.z; e[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = k0 + i < k ? __ldcg(row + k0 + i) : 0.0f;
  }
}

// CTA (r, g): row r < Mp of x (RMS-normalised when norm_w, with the
// statistic of src/ops.cc:55-61 summed in a fixed tree order that every CTA
// of the row repeats identically) over chunks [4 g, 4 g + 4), as fp16 hi (row
// r) and lo (row Mp + r) of the B layout, and the half-block sums (16 inputs,
// the thread's 8 then its lane pair's 8) as the Q4_1 min term's K operand.
// Rows >= rows stage as zero. Each thread takes 8 consecutive inputs.
__global__ void __launch_bounds__(kStageThreads) tc_stage_kernel(const float* x, int ldx, int rows,
                                                                 int k, int chunks,
                                                                 const float* norm_w, float eps,
                                                                 const int* gather, int mp,
                                                                 uint8_t* staged) {
  const int r = blockIdx.x;
  const size_t cb = tc_chunk_bytes(mp);
  __shared__ float part[kStageThreads / 32];
  __shared__ float inv_s;
  pdl_launch_dependents();  // the GEMM after it starts streaming its weights now
  pdl_wait();
  const bool live = r < rows;
  const float* xr = live ? (gather ? x + (size_t)gather[r] * ldx : x + (size_t)r * ldx) : nullptr;
  float inv = 1.0f;
  if (live && norm_w) {
    float ss = 0.0f;
    for (int i = threadIdx.x * 4; i < k; i += kStageThreads * 4) {
      if (i + 3 < k && ((((uintptr_t)(xr + i)) & 15) == 0)) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(xr + i));
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
      } else {
        for (int j = i; j < i + 4 && j < k; ++j) ss = fmaf(xr[j], xr[j], ss);
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int w = 0; w < kStageThreads / 32; ++w) t += part[w];  // fixed order
      t = __fdiv_rn(t, (float)k);
      inv_s = __fdiv_rn(1.0f, sqrtf(__fadd_rn(t, eps)));
    }
    __syncthreads();
    inv = inv_s;
  }
  const int u = blockIdx.y * kStageChunks * 32 + threadIdx.x;  // unit of 8 inputs
  if (u >= chunks * 32) return;  // whole lane pairs leave together
  const int k0 = u * 8;
  float e[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (live) {
    load8(xr, k0, k, e);
    if (norm_w) {
      float w[8];
      load8(norm_w, k0, k, w);
#pragma unroll
      for (int i = 0; i < 8; ++i) e[i] = __fmul_rn(__fmul_rn(e[i], inv), w[i]);
    }
  }
  uint32_t hw[4], lw[4];
  float s = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const __half h0 = __float2half_rn(e[2 * p]), h1 = __float2half_rn(e[2 * p + 1]);
    const __half l0 = __float2half_rn(e[2 * p] - __half2float(h0));
    const __half l1 = __float2half_rn(e[2 * p + 1] - __half2float(h1));
    hw[p] = h2_as_u32(__halves2half2(h0, h1));
    lw[p] = h2_as_u32(__halves2half2(l0, l1));
    s = __fadd_rn(__fadd_rn(s, e[2 * p]), e[2 * p + 1]);
  }
  *reinterpret_cast<uint4*>(staged + staged_off(r, k0, cb)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  *reinterpret_cast<uint4*>(staged + staged_off(mp + r, k0, cb)) =
      make_uint4(lw[0], lw[1], lw[2], lw[3]);
  // half-block sum: the even unit's 8 then the odd unit's 8
  const float s2 = __shfl_xor_sync(0xffffffffu, s, 1);
  if ((u & 1) == 0) {
    const float hs = __fadd_rn(s, s2);
    const __half h = __float2half_rn(hs);
    const __half l = __float2half_rn(hs - __half2float(h));
    const int hb = u >> 1, c = hb >> 4, kk = hb & 15;
    uint8_t* base = staged + (size_t)c * cb + (size_t)mp * 1024 + (size_t)(kk >> 3) * 128 +
                    (size_t)(kk & 7) * 2;
    *reinterpret_cast<__half*>(base + (size_t)(r >> 3) * 256 + (size_t)(r & 7) * 16) = h;
    *reinterpret_cast<__half*>(base + (size_t)((mp + r) >> 3) * 256 + (size_t)((mp + r) & 7) * 16) =
        l;
  }
}

// ---------------------------------------------------------- dequantising

// fp16 hi / lo of d * q (Q4_0: q = code - 8; Q4_1: q = code; Q8_0: q = int8
// code) for a pair of codes given as the magic half2 (bias + code): hi =
// rn(q d), lo = q d - hi, exact (the product has at most 18 significant
// bits). The Q4_1 min m enters through its own MMA against half-block sums of
// x (the kernel's min term), so w = d q + m is never rounded to fp16.
template <int QT>
__device__ __forceinline__ void dq_pair(uint32_t magic, __half2 d2, uint32_t& hi, uint32_t& lo) {
  const __half2 bias = QT == MLB_Q4_0 ? __float2half2_rn(1032.0f)
                                      : (QT == MLB_Q4_1 ? __float2half2_rn(1024.0f)
                                                        : __float2half2_rn(1152.0f));
  const __half2 q = __hsub2(u32_as_h2(magic), bias);
  const __half2 h = __hmul2(q, d2);
  const __half2 l = __hfma2(q, d2, __hneg2(h));
  hi = h2_as_u32(h);
  lo = h2_as_u32(l);
}

// One weight row's GGUF blocks 2 bp and 2 bp + 1 of a super-block as 16 hi
// and 16 lo half2 columns each, in input order (column p holds inputs 2p,
// 2p + 1 of the block); the row is row g + 8 h of the super-block, its codes
// where repack_kernel put them for mma.sync lane g * 4 + cl. Read
// without shared-memory bank conflicts. A warp's 32 rows are rows g + 8 h of
// two super-blocks (jb = 0, 1), and row g's code word for chunk column cl sits
// at bank 16 (g % 2) + 4 cl + 2 (block % 2) + h (super-blocks are a multiple
// of 128 bytes apart): read in the same column order, rows g, g + 2, g + 4,
// g + 6 and the two super-blocks collide (8 ways). So row g reads column
// (i + g / 2) % 4 at step i, and super-block 1 reads the pair's blocks in
// swapped order; selects put the words back in (block, column) order.
template <int QT>
__device__ __forceinline__ void dq_block_pair(const uint8_t* sb, int g, int h, int jb, int bp,
                                              uint32_t (&hv)[2][16], uint32_t (&lv)[2][16]) {
  constexpr int qbytes = QT == MLB_Q8_0 ? 4096 : 2048;
  const int r = (g >> 1) & 3;
  constexpr int W = QT == MLB_Q8_0 ? 2 : 1;  // 32-bit code words per (block, column, row)
  uint32_t w[2][4][W];                       // [block parity][column][word]
  {
    uint32_t t[4][2][W];  // [step][pair slot][word]: block 2 bp + (slot ^ jb), column (i + r) % 4
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int cl = (i + r) & 3;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int b = 2 * bp + (p ^ jb);
        if (QT == MLB_Q8_0) {
          const uint2 v = *reinterpret_cast<const uint2*>(sb + (size_t)(b * 32 + g * 4 + cl) * 16 + h * 8);
          t[i][p][0] = v.x;
          t[i][p][W - 1] = v.y;
        } else {
          t[i][p][0] = *reinterpret_cast<const uint32_t*>(
              sb + (size_t)(bp * 32 + g * 4 + cl) * 16 + (b & 1) * 8 + h * 4);
        }
      }
    }
#pragma unroll
    for (int P = 0; P < 2; ++P)
#pragma unroll
      for (int k = 0; k < W; ++k) {
        uint32_t u[4], v1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) u[i] = jb ? t[i][P ^ 1][k] : t[i][P][k];
        // column cl was read at step (cl - r) % 4
#pragma unroll
        for (int c = 0; c < 4; ++c) v1[c] = (r & 1) ? u[(c + 3) & 3] : u[c];
#pragma unroll
        for (int c = 0; c < 4; ++c) w[P][c][k] = (r & 2) ? v1[(c + 2) & 3] : v1[c];
      }
  }
#pragma unroll
  for (int P = 0; P < 2; ++P) {
    const int b = 2 * bp + P;
    const uint8_t* sc = sb + qbytes + (g * 8 + b) * 4 + 2 * h;
    const __half d = __ushort_as_half(*reinterpret_cast<const unsigned short*>(sc));
    const __half2 d2 = __halves2half2(d, d);
#pragma unroll
    for (int cl = 0; cl < 4; ++cl) {
      uint32_t mg[4];
      if (QT == MLB_Q8_0) {
        const uint32_t xa = w[P][cl][0] ^ 0x80808080u, xb = w[P][cl][W - 1] ^ 0x80808080u;
        mg[0] = __byte_perm(xa, 0x64646464u, 0x4140);  // inputs 2cl, 2cl + 1
        mg[1] = __byte_perm(xa, 0x64646464u, 0x4342);  // 2cl + 8, 2cl + 9
        mg[2] = __byte_perm(xb, 0x64646464u, 0x4140);  // 2cl + 16, 2cl + 17
        mg[3] = __byte_perm(xb, 0x64646464u, 0x4342);  // 2cl + 24, 2cl + 25
      } else {
        const uint32_t x = w[P][cl][0];
        const uint32_t M1 = 0x000F000Fu, E = 0x64006400u;
        mg[0] = lop3_and_or(x, M1, E);        // low nibbles of bytes 0, 2: inputs 2cl, 2cl + 1
        mg[1] = lop3_and_or(x >> 8, M1, E);   // bytes 1, 3: 2cl + 8, 2cl + 9
        mg[2] = lop3_and_or(x >> 4, M1, E);   // high nibbles of 0, 2: 2cl + 16, 2cl + 17
        mg[3] = lop3_and_or(x >> 12, M1, E);  // high nibbles of 1, 3: 2cl + 24, 2cl + 25
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) dq_pair<QT>(mg[e], d2, hv[P][4 * e + cl], lv[P][4 * e + cl]);
    }
  }
}

// Q4_1: the min of block b of this row, duplicated as (m, m): one TMEM
// column of the min term's A operand, whose K runs over the chunk's 16
// half-blocks (half-block 2b and 2b + 1 both belong to block b).
__device__ __forceinline__ uint32_t q41_min_pair(const uint8_t* sb, int g, int h, int b) {
  const unsigned short m =
      *reinterpret_cast<const unsigned short*>(sb + 2304 + (g * 8 + b) * 4 + 2 * h);
  return (uint32_t)m | ((uint32_t)m << 16);
}

__device__ __forceinline__ void tmem_st2(uint32_t taddr, uint32_t v0, uint32_t v1) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(v0),
               "r"(v1)
               : "memory");
}

// ------------------------------------------------------ work partition

// Unit u = tile * C + chunk; CTA i of G owns units [floor(i U / G),
// floor((i + 1) U / G)). The first CTA boundary strictly after unit x is
// boundary k = ceil((x + 1) G / U).
__host__ __device__ inline long long first_boundary_after(long long x, long long U, long long G) {
  return ((x + 1) * G + U - 1) / U;
}
__host__ __device__ inline long long boundary(long long k, long long U, long long G) {
  return k * U / G;
}
// Number of runs of tile rt (its chunks cut by CTA boundaries).
__host__ __device__ inline int tile_runs(long long rt, long long C, long long U, long long G) {
  const long long k0 = first_boundary_after(rt * C, U, G);
  const long long k1 = first_boundary_after((rt + 1) * C - 1, U, G);  // first at or past the end
  return 1 + (int)(k1 - k0);
}
__host__ __device__ inline int max_tile_runs(long long C, long long U, long long G) {
  return (int)((C * G + U - 1) / U) + 2;
}

struct TcArgs {
  const uint8_t* w;  // super-blocks
  int sbb, ntiles, nchunks, gc;
  const uint8_t* staged;
  int rows;
  int stages, stage_bytes, sb_region;
  float* ws;
  int* counters;  // [row tiles][8 warp slices]
  int maxruns;
  DeviceStatus* status;
  BEpi epi;
};

struct TcShared {
  uint64_t full[kMaxRingStages], empty[kMaxRingStages];
  uint64_t afull[2], aempty[2], dfull, dempty, fin;
  uint32_t tmem_base;
  int abort_flag;
};

// Bounded mbarrier wait that also gives up when another thread aborted.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, TcShared& sh,
                                        DeviceStatus* st, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*(volatile int*)&sh.abort_flag) return false;
    if (clock64() - t0 > kTcWaitCycles) {
      if (atomicCAS(&st->code, 0, MLB_ERR_TIMEOUT) == 0) atomicExch(&st->where, where);
      *(volatile int*)&sh.abort_flag = 1;
      return false;
    }
  }
  return true;
}

// One KV-cache element: fp32, or bf16 rounded to nearest even.
__device__ __forceinline__ void kv_store(float* base, int bf16, size_t i, float v) {
  if (bf16)
    reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else
    base[i] = v;
}

// The fused epilogue of one warp slice: rows n (this lane's) of a tile and
// batch columns cbase .. cbase + NC - 1, values v.
template <int NC>
__device__ __forceinline__ void tc_epilogue(const BEpi& e, int n, int lr, int lane, int cbase,
                                            const float (&v)[NC]) {
  if (e.kind == kEpiSwiglu) {
    // tile rows 0..7 are gate rows, 8..15 the matching up rows (lane + 8)
    const int hrow = (n >> 4) * 8 + (lr & 7);
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const float up = __shfl_down_sync(0xffffffffu, v[i], 8);
      const int r = cbase + i;
      if ((lr & 15) < 8 && r < e.rows && hrow < e.n_out) {
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v[i])));
        e.y[(size_t)r * e.ldy + hrow] = __fmul_rn(__fmul_rn(v[i], sg), up);
      }
    }
    return;
  }
  if (e.kind == kEpiQkv) {
    int local, size, sec;
    if (n < e.k_off) {
      sec = 0; local = n; size = e.q_rows;
    } else if (n < e.v_off) {
      sec = 1; local = n - e.k_off; size = e.kv_rows;
    } else {
      sec = 2; local = n - e.v_off; size = e.kv_rows;
    }
    const int D = e.head_dim;
    auto logical = [&](int l) {
      if (!e.neox || sec == 2) return l;
      const int hd = l / D, qd = l - hd * D;
      return hd * D + ((qd & 1) ? (qd >> 1) + D / 2 : (qd >> 1));
    };
    const int bias_base = sec == 0 ? 0 : (sec == 1 ? e.q_rows : e.q_rows + e.kv_rows);
    const bool live = local < size;
    const int L = live ? logical(local) : 0;
    const int Lp = live ? logical(local ^ 1) : 0;
    const float bv = (live && e.bias) ? e.bias[bias_base + L] : 0.0f;
    const float bp = (live && e.bias) ? e.bias[bias_base + Lp] : 0.0f;
    const int in_head = L % D;
    bool first;
    int jj;
    if (e.neox) {
      first = in_head < D / 2;
      jj = first ? in_head : in_head - D / 2;
    } else {
      first = (in_head & 1) == 0;
      jj = in_head >> 1;
    }
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[i], 1);
      const int r = cbase + i;
      if (!live || r >= e.rows) continue;
      const float val = e.bias ? __fadd_rn(v[i], bv) : v[i];
      const int pos = e.row_pos[r];
      const int seq = e.row_seq ? e.row_seq[r] : r;
      if (sec == 2) {
        kv_store(e.values, e.kv_bf16, (size_t)seq * e.seq_stride + (size_t)pos * e.kv_rows + L, val);
        continue;
      }
      // rotation of (this, partner) as src/ops.cc:155-156 / 174-175
      const float w = e.bias ? __fadd_rn(partner, bp) : partner;
      const float2 cs = e.rope[(size_t)pos * (D / 2) + jj];
      const float out = first ? __fsub_rn(__fmul_rn(val, cs.x), __fmul_rn(w, cs.y))
                              : __fadd_rn(__fmul_rn(w, cs.y), __fmul_rn(val, cs.x));
      if (sec == 0)
        e.q_out[(size_t)r * e.q_rows + L] = out;
      else
        kv_store(e.keys, e.kv_bf16, (size_t)seq * e.seq_stride + (size_t)pos * e.kv_rows + L, out);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int r = cbase + i;
    const bool ok = r < e.rows && n < e.n_out;
    if (ok) {
      if (e.kind == kEpiResidual)
        e.y[(size_t)r * e.ldy + n] = __fadd_rn(__ldcg(e.resid + (size_t)r * e.ldr + n), v[i]);
      else
        e.y[(size_t)r * e.ldy + n] = v[i];
    }
    if (e.kind == kEpiStore && e.argmax_keys) {
      unsigned long long key = ok ? argmax_key_of(v[i], e.argmax_base + n) : 0ull;
      key = warp_max_u64(key);
      if (lane == 0 && key) atomicMax(&e.argmax_keys[r], key);
    }
  }
}

template <int QT, int MP>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const TcArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  TcShared& sh = *reinterpret_cast<TcShared*>(smem);
  uint8_t* ring = smem + 1024;
  constexpr int NC = MP / 2;  // batch columns of one epilogue warp
  // staged chunk stride in global memory, and the bytes a stage copies (the
  // half-block sums only for the Q4_1 min term)
  constexpr uint32_t kChunkStride = (uint32_t)MP * 1088u;
  constexpr uint32_t kChunkBytes = (uint32_t)MP * (QT == MLB_Q4_1 ? 1088u : 1024u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long C = a.nchunks;
  const long long RT = (a.ntiles + 7) / 8;
  const long long U = RT * C, G = gridDim.x;
  const long long u_begin = boundary(blockIdx.x, U, G), u_end = boundary(blockIdx.x + 1, U, G);

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sh.afull[t], kDqWarps);
      mbar_init(&sh.aempty[t], 1);
    }
    mbar_init(&sh.dfull, 1);
    mbar_init(&sh.dempty, kDqWarps);
    mbar_init(&sh.fin, 1);
    sh.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sh.tmem_base;

  pdl_launch_dependents();  // dependents still wait for this grid to complete
  if (warp == 0) {
    // ------------------------------------------------------ producer
    if (lane == 0) {
      long long it = 0;
      long long last_it[kMaxRingStages];
      for (int s = 0; s < kMaxRingStages; ++s) last_it[s] = -1;
      auto issue_weights = [&](long long u, int s) {
        const int rt = (int)(u / C), c = (int)(u - (long long)rt * C);
        uint8_t* st = ring + (size_t)s * a.stage_bytes;
        const int nt = min(8, a.ntiles - rt * 8);
        mbar_arrive_expect_tx(&sh.full[s], (uint32_t)(nt * a.sbb) + kChunkBytes);
        for (int j = 0; j < nt; ++j) {
          const long long sbi = sb_index(rt * 8 + j, c, a.ntiles, a.nchunks, a.gc);
          bulk_g2s(st + j * a.sbb, a.w + sbi * a.sbb, a.sbb, &sh.full[s]);
        }
      };
      auto issue_acts = [&](long long u, int s) {
        const int c = (int)(u % C);
        uint8_t* st = ring + (size_t)s * a.stage_bytes;
        bulk_g2s(st + a.sb_region, a.staged + (size_t)c * kChunkStride, kChunkBytes, &sh.full[s]);
      };
      // the first stages' weights do not depend on the previous kernel:
      // stream them while it finishes (programmatic dependent launch), then
      // wait for it before copying the activations it staged
      const long long pre = min((long long)a.stages, u_end - u_begin);
      for (long long i = 0; i < pre; ++i) issue_weights(u_begin + i, (int)i);
      pdl_wait();
      for (long long i = 0; i < pre; ++i) {
        issue_acts(u_begin + i, (int)i);
        last_it[i] = i;
      }
      it = pre;
      for (long long u = u_begin + pre; u < u_end; ++u, ++it) {
        const int s = (int)(it % a.stages);
        const uint32_t par = (uint32_t)((it / a.stages) & 1);
        if (!tc_wait(&sh.empty[s], par ^ 1u, sh, a.status, 700)) break;
        issue_weights(u, s);
        issue_acts(u, s);
        last_it[s] = it;
      }
      if (*(volatile int*)&sh.abort_flag) {
        // copies still landing in the ring: wait for each stage's last phase
        for (int s = 0; s < a.stages; ++s) {
          if (last_it[s] < 0) continue;
          const uint32_t par = (uint32_t)((last_it[s] / a.stages) & 1);
          const long long t0 = clock64();
          while (!mbar_try_wait(&sh.full[s], par))
            if (clock64() - t0 > kTcWaitCycles) break;
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t d_t = tbase + kDCol;
      constexpr uint32_t id2 = idesc_f16(2 * MP), id1 = idesc_f16(MP);
      // ring stage of the next unit and its phase parity, kept as counters
      // (no 64-bit division between units: this thread's issue rate bounds
      // the kernel)
      int s = 0;
      uint32_t sph = 0u;
      long long ait = 0, rit = 0;
      bool ok = true;
      for (long long u = u_begin; u < u_end && ok; ++rit) {
        const long long rt = u / C;
        const long long run_end = min(u_end, (rt + 1) * C);
        if (!tc_wait(&sh.dempty, (uint32_t)((rit & 1) ^ 1), sh, a.status, 710)) break;
        tc_fence_after();
        bool first = true;
        for (; u < run_end && ok; ++u) {
          if (!tc_wait(&sh.full[s], sph, sh, a.status, 711)) {
            ok = false;
            break;
          }
          const uint32_t bbase = smem_addr(ring + (size_t)s * a.stage_bytes + a.sb_region);
          for (int kh = 0; kh < 2 && ok; ++kh, ++ait) {
            const int t = (int)(ait & 1);
            if (!tc_wait(&sh.afull[t], (uint32_t)((ait >> 1) & 1), sh, a.status, 712)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_hi = tbase + t * kAStageCols, a_lo = a_hi + 64;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint64_t bd = smem_desc(bbase + (uint32_t)(kh * 16 + 2 * ks) * 128u, 4096u);
              tc_mma_ts(d_t, a_hi + 8 * ks, bd, id2, first ? 0u : 1u);
              tc_mma_ts(d_t, a_lo + 8 * ks, bd, id1, 1u);
              first = false;
            }
            if (QT == MLB_Q4_1 && kh == 1) {
              // the chunk's min term: sum over blocks of m * (block sum of x),
              // A = the mins (TMEM columns 384..391), B = half-block sums
              const uint64_t bm = smem_desc(bbase + (uint32_t)MP * 1024u, 256u);
              tc_mma_ts(d_t, tbase + kMinCol, bm, id2, 1u);
            }
            tc_commit(&sh.aempty[t]);
          }
          if (!ok) break;
          tc_commit(&sh.empty[s]);
          if (++s == a.stages) {
            s = 0;
            sph ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&sh.dfull);
      }
      // every MMA this thread issued has completed before TMEM is released
      tc_commit(&sh.fin);
      const long long t0 = clock64();
      while (!mbar_try_wait(&sh.fin, 0))
        if (clock64() - t0 > kTcWaitCycles) break;
    }
  } else {
    // ------------------------------------------- dequantise + epilogue
    pdl_wait();  // the epilogue reads and writes the previous kernels' data
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int slice = warp - 2;
    const int lr = 32 * q + lane;  // weight row within the CTA tile (TMEM lane)
    const int j = lr >> 4, r16 = lr & 15, g = r16 & 7, h = r16 >> 3;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    const int cbase = half * NC;
    int s = 0;  // ring stage of the next unit and its phase parity
    uint32_t sph = 0u;
    long long ait = 0, rit = 0;
    bool ok = true;
    for (long long u = u_begin; u < u_end && ok; ++rit) {
      const long long rt = u / C;
      const long long run_start = u;
      const long long run_end = min(u_end, (rt + 1) * C);
      for (; u < run_end && ok; ++u) {
        if (!__all_sync(0xffffffffu, tc_wait(&sh.full[s], sph, sh, a.status, 720))) {
          ok = false;
          break;
        }
        const uint8_t* sb = ring + (size_t)s * a.stage_bytes + (size_t)j * a.sbb;
        if (++s == a.stages) {
          s = 0;
          sph ^= 1u;
        }
        const bool valid = rt * 8 + j < a.ntiles;
        for (int kh = 0; kh < 2; ++kh, ++ait) {
          const int t = (int)(ait & 1);
          if (!__all_sync(0xffffffffu, tc_wait(&sh.aempty[t], (uint32_t)(((ait >> 1) & 1) ^ 1), sh,
                                               a.status, 721))) {
            ok = false;
            break;
          }
          {
            // blocks 4 kh + 2 half + bb of the chunk: block pair 2 kh + half
            uint32_t hv[2][16], lv[2][16];
            if (valid) {
              dq_block_pair<QT>(sb, g, h, j & 1, 2 * kh + half, hv, lv);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) hv[0][i] = lv[0][i] = hv[1][i] = lv[1][i] = 0u;
            }
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
              const uint32_t col = tbase + lane_base + t * kAStageCols + 16 * (2 * half + bb);
              tmem_st16(col, hv[bb]);
              tmem_st16(col + 64, lv[bb]);
            }
          }
          if (QT == MLB_Q4_1 && kh == 1) {
            // the mins of this warp's blocks {2 half, 2 half + 1, 4 + 2 half, 5 + 2 half}
#pragma unroll
            for (int p = 0; p < 2; ++p) {
              const int b0 = 4 * p + 2 * half;
              const uint32_t m0 = valid ? q41_min_pair(sb, g, h, b0) : 0u;
              const uint32_t m1 = valid ? q41_min_pair(sb, g, h, b0 + 1) : 0u;
              tmem_st2(tbase + lane_base + kMinCol + b0, m0, m1);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.afull[t]);
        }
      }
      if (!ok) break;
      // the run's accumulator: hi columns [0, MP) plus lo columns [MP, 2 MP)
      if (!__all_sync(0xffffffffu, tc_wait(&sh.dfull, (uint32_t)(rit & 1), sh, a.status, 722)))
        break;
      tc_fence_after();
      float v[NC];
#pragma unroll
      for (int c8 = 0; c8 < NC / 8; ++c8) {
        uint32_t hw[8], lw[8];
        tmem_ld8(tbase + lane_base + kDCol + cbase + 8 * c8, hw);
        tmem_ld8(tbase + lane_base + kDCol + MP + cbase + 8 * c8, lw);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[8 * c8 + i] = __uint_as_float(hw[i]) + __uint_as_float(lw[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.dempty);
      const int n = (int)rt * kTcRows + lr;
      const bool whole = run_start == rt * C && run_end == (rt + 1) * C;
      if (!whole) {
        // this warp slice's partial into its run slot; the last of the
        // tile's runs to finish this slice sums the slots in chunk order
        // slot layout [run][column][row]: a warp's 32 rows of one column are
        // one coalesced 128-byte line
        const long long k0 = first_boundary_after(rt * C, U, G);
        const int jr = run_start == rt * C ? 0 : (int)(blockIdx.x - k0 + 1);
        float* slot = a.ws + (((size_t)rt * a.maxruns + jr) * MP + cbase) * kTcRows + lr;
#pragma unroll
        for (int i = 0; i < NC; ++i) slot[(size_t)i * kTcRows] = v[i];
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          const int nr = tile_runs(rt, C, U, G);
          last = atomicAdd(&a.counters[rt * 8 + slice], 1) == nr - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        const int nr = tile_runs(rt, C, U, G);
#pragma unroll
        for (int i = 0; i < NC; ++i) v[i] = 0.0f;
        for (int jj = 0; jj < nr; ++jj) {
          const float* sl = a.ws + (((size_t)rt * a.maxruns + jj) * MP + cbase) * kTcRows + lr;
#pragma unroll
          for (int i = 0; i < NC; ++i) v[i] += __ldcg(sl + (size_t)i * kTcRows);
        }
        if (lane == 0) a.counters[rt * 8 + slice] = 0;
      }
      tc_epilogue<NC>(a.epi, n, lr, lane, cbase, v);
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tbase, kTmemCols);
}

template <int QT>
void* tc_kernel_for(int mp) {
  switch (mp) {
    case 16: return (void*)tc_gemm_kernel<QT, 16>;
    case 32: return (void*)tc_gemm_kernel<QT, 32>;
    case 48: return (void*)tc_gemm_kernel<QT, 48>;
    case 64: return (void*)tc_gemm_kernel<QT, 64>;
    default: invalid("tensor-core GEMM: no kernel for " + std::to_string(mp) + " padded rows");
  }
}

}  // namespace

void tc_stage_launch(const float* x, int ldx, int rows, int k, int chunks, const float* norm_w,
                     float eps, const int* gather, uint8_t* staged, cudaStream_t stream,
                     bool pdl) {
  const int mp = tc_mp(rows);
  if (mp > kTcMaxMp) invalid("tensor-core GEMM: more than 64 activation rows per pass");
  const dim3 grid(mp, (chunks + kStageChunks - 1) / kStageChunks);
  launch_pdl(tc_stage_kernel, grid, dim3(kStageThreads), 0, stream, pdl, x, ldx, rows, k, chunks,
             norm_w, eps, gather, mp, staged);
}

// CTAs of a launch: at most one per (tile, chunk) unit, so that every CTA
// owns at least one unit and the CTA boundaries are distinct.
static int tc_grid(const QMatrix& m, int grid) {
  const long long U = (long long)((m.ntiles + 7) / 8) * m.nchunks;
  return (int)std::max(1LL, std::min<long long>(grid, U));
}

size_t tc_partial_floats(const QMatrix& m, int rows, int grid) {
  grid = tc_grid(m, grid);
  const long long C = m.nchunks, RT = (m.ntiles + 7) / 8, U = RT * C;
  const int mr = max_tile_runs(C, U, grid);
  return (size_t)RT * mr * kTcRows * tc_mp(rows);
}

int tc_counter_count(const QMatrix& m) { return (m.ntiles + 7) / 8 * 8; }

bool tc_gemm_ok(const QMatrix& m, int rows) {
  return (m.qtype == MLB_Q4_0 || m.qtype == MLB_Q4_1 || m.qtype == MLB_Q8_0) && rows >= 1 &&
         tc_mp(rows) <= kTcMaxMp;
}

void tc_gemm_launch(const QMatrix& m, const uint8_t* staged, int rows, const BEpi& epi,
                    const TcWorkspace& ws, cudaStream_t stream, int grid_ctas, bool pdl) {
  if (!tc_gemm_ok(m, rows)) invalid("tensor-core GEMM: unsupported matrix or batch");
  int dev = 0;
  MLB_CUDA(cudaGetDevice(&dev));
  const int grid = tc_grid(m, grid_ctas > 0 ? grid_ctas : sm_count(dev));
  const int mp = tc_mp(rows);
  TcArgs a{};
  a.w = m.data;
  a.sbb = sb_bytes(m.qtype);
  a.ntiles = m.ntiles;
  a.nchunks = m.nchunks;
  a.gc = m.gc;
  a.staged = staged;
  a.rows = rows;
  a.sb_region = (8 * a.sbb + 127) / 128 * 128;
  a.stage_bytes = a.sb_region + (int)tc_chunk_bytes(mp);
  constexpr int kSmemBudget = 220 * 1024;
  a.stages = std::min(kMaxRingStages, (kSmemBudget - 1024) / a.stage_bytes);
  if (a.stages < 2) invalid("tensor-core GEMM: ring does not fit in shared memory");
  const long long C = m.nchunks, RT = (m.ntiles + 7) / 8, U = RT * C;
  a.maxruns = max_tile_runs(C, U, grid);
  if (ws.partial_floats < tc_partial_floats(m, rows, grid) ||
      ws.counter_count < tc_counter_count(m))
    invalid("tensor-core GEMM: workspace too small");
  a.ws = ws.partials;
  a.counters = ws.counters;
  a.status = ws.status;
  a.epi = epi;
  a.epi.rows = rows;
  const size_t smem = 1024 + (size_t)a.stages * a.stage_bytes;
  void* fn = m.qtype == MLB_Q4_0 ? tc_kernel_for<MLB_Q4_0>(mp)
                                 : (m.qtype == MLB_Q4_1 ? tc_kernel_for<MLB_Q4_1>(mp)
                                                        : tc_kernel_for<MLB_Q8_0>(mp));
  MLB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void* params[] = {&a};
  MLB_CUDA(cudaLaunchKernelExC(&cfg, fn, params));
}

}  // namespace mlb

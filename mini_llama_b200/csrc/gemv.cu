// gemv.cu — quantised GEMV kernels for the decode path.
//
// Reference: the per-output sequential loops of Q80/Q40/Q41LinearKernel
// (src/cuda_quant.cu:36-130) and of the CPU LinearQuantizedImpl
// (src/quant.cc:365-425). Dequantisation follows the CPU definition
// (src/quant.cc:430-456): Q8_0 w = d*q, Q4_0 w = d*(q-8), Q4_1 w = d*q + m
// (the reference GPU kernel's d*m*q for Q4_1 is not followed).
//
// How a super-block (16 rows x 256 k) is computed (one warp):
//  * The 4-bit / 8-bit codes are turned into exact fp16 values (q-8, q or the
//    int8) with the magic-exponent trick: OR the code into the mantissa of
//    1024.0h and subtract (lop3 + hsub2/hfma2); no int->float conversions.
//  * x is split once into fp16 hi + lo parts (x = hi + lo to ~22 bits), which
//    sit in columns 2r and 2r+1 of the mma B operand for batch row r, so one
//    m16n8k16 MMA yields hi and lo partial dots of 16 rows for up to 4 rows
//    of x. Products of an exact 4/8-bit code and an fp16 value are exact in
//    the fp32 accumulator.
//  * Per 32-input block the fp32 block dot is scaled by the fp16 block scale
//    (and for Q4_1 the min times the block sum of x is added).
// The weight stream is fed by cp.async.bulk copies into a per-warp shared
// memory ring; the first copies are issued before griddepcontrol.wait, so with
// programmatic dependent launch a GEMV streams its weights while the previous
// kernel finishes.
#include "gemv.cuh"
#include "gemv_dev.cuh"

#include <algorithm>
#include <cmath>
#include <vector>

namespace mlb {

// ----------------------------------------------------------------- geometry

void qmatrix_geometry(QMatrix& m, int qtype, int n, int k, int max_batch) {
  if (n <= 0 || k <= 0) invalid("qmatrix: empty tensors are not supported");
  m.qtype = qtype;
  m.n = n;
  m.k = k;
  m.ntiles = (n + kTileRows - 1) / kTileRows;
  m.gguf_bytes = (size_t)n * gguf_row_bytes(qtype, k);
  if (qtype == MLB_F32) {
    m.nchunks = 0;
    m.gc = 0;
    m.ngroups = 0;
    m.nsb = 0;
    m.bytes = (size_t)m.ntiles * kTileRows * (size_t)k * 4;
    return;
  }
  if (qtype != MLB_Q8_0 && qtype != MLB_Q4_0 && qtype != MLB_Q4_1)
    invalid("qmatrix: unsupported quant type " + std::to_string(qtype));
  m.nchunks = (k + kChunkK - 1) / kChunkK;
  // Chunk group: all of K in one group up to 64 chunks (K <= 16384) for one
  // batch row (the staged activations then take at most 72 KB of shared
  // memory); wider batches stage proportionally fewer chunks, and Q8_0 (whose
  // weight ring needs twice the room) half as many again.
  const int mb = max_batch < 1 ? 1 : (max_batch > kMaxBatch ? kMaxBatch : max_batch);
  const int mbucket = mb >= 3 ? 4 : mb;
  const int whole = mbucket == 1 ? 64 : (qtype == MLB_Q8_0 ? 32 : 64) / mbucket;
  m.gc = m.nchunks <= whole ? m.nchunks : whole / 2;
  m.ngroups = (m.nchunks + m.gc - 1) / m.gc;
  m.nsb = (long long)m.ntiles * m.nchunks;
  m.bytes = (size_t)m.nsb * sb_bytes(qtype);
}


// ------------------------------------------------------------------- repack

// One thread per (tile, chunk, block-in-chunk, lane).
__global__ void repack_kernel(int qtype, uint8_t* dst, int ntiles, int nchunks, int gc, int n,
                              int kblocks, const uint8_t* src, size_t src_pitch,
                              const int* row_map, int col_block0) {
  long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)ntiles * nchunks * 8 * 32;
  if (tid >= total) return;
  int lane = (int)(tid & 31);
  int b = (int)((tid >> 5) & 7);
  long long tc = tid >> 8;
  int c = (int)(tc % nchunks);
  int t = (int)(tc / nchunks);
  int g = lane >> 2, cl = lane & 3;
  int sbb = qtype == MLB_Q8_0 ? 4352 : (qtype == MLB_Q4_1 ? 2560 : 2304);
  uint8_t* sb = dst + sb_index(t, c, ntiles, nchunks, gc) * sbb;
  int blk = c * 8 + b;
  int bsz = qtype == MLB_Q8_0 ? 34 : (qtype == MLB_Q4_1 ? 20 : 18);
  const uint8_t* rowsrc[2] = {nullptr, nullptr};
  for (int h = 0; h < 2; ++h) {
    int R = t * 16 + g + 8 * h;
    int sr = row_map ? (R < n ? row_map[R] : -1) : (R < n ? R : -1);
    if (sr >= 0 && blk < kblocks)
      rowsrc[h] = src + (size_t)sr * src_pitch + (size_t)(col_block0 + blk) * bsz;
  }
  if (qtype == MLB_Q8_0) {
    uint8_t out[16];
    for (int h = 0; h < 2; ++h) {
      const uint8_t* q = rowsrc[h] ? rowsrc[h] + 2 : nullptr;
      const int ks[8] = {2 * cl, 2 * cl + 1, 2 * cl + 8, 2 * cl + 9,
                         2 * cl + 16, 2 * cl + 17, 2 * cl + 24, 2 * cl + 25};
      for (int i = 0; i < 8; ++i) out[h * 8 + i] = q ? q[ks[i]] : 0;
    }
    uint8_t* o = sb + (size_t)(b * 32 + lane) * 16;
    for (int i = 0; i < 16; ++i) o[i] = out[i];
  } else {
    int qoff = qtype == MLB_Q4_1 ? 4 : 2;
    uint8_t out[8];
    for (int h = 0; h < 2; ++h) {
      const uint8_t* q = rowsrc[h] ? rowsrc[h] + qoff : nullptr;
      const int js[4] = {2 * cl, 2 * cl + 8, 2 * cl + 1, 2 * cl + 9};
      for (int i = 0; i < 4; ++i) out[h * 4 + i] = q ? q[js[i]] : 0;
    }
    // [block pair p][lane][16 B]: block 2p in bytes 0..7, block 2p+1 in 8..15
    uint8_t* o = sb + (size_t)((b >> 1) * 32 + lane) * 16 + (b & 1) * 8;
    for (int i = 0; i < 8; ++i) o[i] = out[i];
  }
  if (cl == 0) {
    int qbytes = qtype == MLB_Q8_0 ? 4096 : 2048;
    uint8_t* s = sb + qbytes + (g * 8 + b) * 4;
    for (int h = 0; h < 2; ++h) {
      const uint8_t* r = rowsrc[h];
      s[2 * h] = r ? r[0] : 0;
      s[2 * h + 1] = r ? r[1] : 0;
    }
    if (qtype == MLB_Q4_1) {
      uint8_t* mm = sb + 2304 + (g * 8 + b) * 4;
      for (int h = 0; h < 2; ++h) {
        const uint8_t* r = rowsrc[h];
        mm[2 * h] = r ? r[2] : 0;
        mm[2 * h + 1] = r ? r[3] : 0;
      }
    }
  }
}

// F32 weights: rows padded to a multiple of 16, same row order as the source.
__global__ void repack_f32_kernel(float* dst, int npad, int n, int k, const uint8_t* src,
                                  size_t src_pitch, const int* row_map, int col0) {
  long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= (long long)npad * k) return;
  int R = (int)(tid / k), c = (int)(tid % k);
  int sr = row_map ? (R < n ? row_map[R] : -1) : (R < n ? R : -1);
  dst[tid] = sr >= 0 ? reinterpret_cast<const float*>(src + (size_t)sr * src_pitch)[col0 + c]
                     : 0.0f;
}

void qmatrix_repack(const QMatrix& m, const uint8_t* src, size_t src_pitch, const int* row_map,
                    int col_block0, cudaStream_t stream) {
  if (m.qtype == MLB_F32) {
    long long total = (long long)m.ntiles * kTileRows * m.k;
    repack_f32_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
        reinterpret_cast<float*>(m.data), m.ntiles * kTileRows, m.n, m.k, src, src_pitch,
        row_map, col_block0 * 32);
  } else {
    long long total = (long long)m.ntiles * m.nchunks * 256;
    repack_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
        m.qtype, m.data, m.ntiles, m.nchunks, m.gc, m.n, (m.k + 31) / 32, src, src_pitch,
        row_map, col_block0);
  }
  MLB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------ dequant

// Dequantised weights straight from the repacked super-block layout: one
// thread per (row, GGUF block) of the logical [n, k] matrix reads the codes
// and scales where the GEMV's lanes read them (repack_kernel's placement) and
// decodes each 4-bit code through the same magic-exponent half (1024 + q),
// then forms the value as DequantizeFromQ40/Q41/Q80 do (src/quant.cc:170-361):
// Q4_0 (q - 8) * d, Q4_1 q * d + m (product and sum each rounded), Q8_0
// d * q. Inputs past k are not written.
__global__ void dequant_sb_kernel(int qtype, const uint8_t* sbs, int ntiles, int nchunks, int gc,
                                  int n, int k, float* out) {
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int kb = (k + 31) / 32;
  if (tid >= (long long)n * kb) return;
  const int R = (int)(tid / kb), blk = (int)(tid - (long long)R * kb);
  const int t = R >> 4, r16 = R & 15, g = r16 & 7, h = r16 >> 3;
  const int c = blk >> 3, b = blk & 7;
  const int sbb = qtype == MLB_Q8_0 ? 4352 : (qtype == MLB_Q4_1 ? 2560 : 2304);
  const int qbytes = qtype == MLB_Q8_0 ? 4096 : 2048;
  const uint8_t* sb = sbs + sb_index(t, c, ntiles, nchunks, gc) * sbb;
  const uint8_t* sc = sb + qbytes + (g * 8 + b) * 4 + 2 * h;
  const float d = __half2float(__ushort_as_half((unsigned short)(sc[0] | (sc[1] << 8))));
  float m = 0.0f;
  if (qtype == MLB_Q4_1) {
    const uint8_t* mm = sb + 2304 + (g * 8 + b) * 4 + 2 * h;
    m = __half2float(__ushort_as_half((unsigned short)(mm[0] | (mm[1] << 8))));
  }
  float* o = out + (size_t)R * k + (size_t)blk * 32;
  const int nv = min(32, k - blk * 32);
  for (int cl = 0; cl < 4; ++cl) {
    const int lane = g * 4 + cl;
    if (qtype == MLB_Q8_0) {
      const int8_t* q = reinterpret_cast<const int8_t*>(sb + (size_t)(b * 32 + lane) * 16 + h * 8);
      const int ks[8] = {2 * cl, 2 * cl + 1, 2 * cl + 8, 2 * cl + 9,
                         2 * cl + 16, 2 * cl + 17, 2 * cl + 24, 2 * cl + 25};
      for (int i = 0; i < 8; ++i)
        if (ks[i] < nv) o[ks[i]] = __fmul_rn(d, (float)q[i]);
    } else {
      const uint8_t* q = sb + (size_t)((b >> 1) * 32 + lane) * 16 + (b & 1) * 8 + h * 4;
      const int js[4] = {2 * cl, 2 * cl + 8, 2 * cl + 1, 2 * cl + 9};
      for (int i = 0; i < 4; ++i) {
        for (int hi = 0; hi < 2; ++hi) {
          const int pos = js[i] + 16 * hi;
          if (pos >= nv) continue;
          const unsigned nib = hi ? (q[i] >> 4) : (q[i] & 15u);
          const float code = __half2float(__ushort_as_half((unsigned short)(0x6400u | nib)));
          if (qtype == MLB_Q4_0)
            o[pos] = __fmul_rn(__fsub_rn(code, 1032.0f), d);
          else
            o[pos] = __fadd_rn(__fmul_rn(__fsub_rn(code, 1024.0f), d), m);
        }
      }
    }
  }
}

void qmatrix_dequant(const QMatrix& m, float* out, cudaStream_t stream) {
  if (m.qtype == MLB_F32) invalid("mlb_qmatrix_dequant: F32 weights have no quantised form");
  const long long total = (long long)m.n * ((m.k + 31) / 32);
  if (total == 0) return;
  dequant_sb_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
      m.qtype, m.data, m.ntiles, m.nchunks, m.gc, m.n, m.k, out);
  MLB_CUDA(cudaGetLastError());
}

// ---------------------------------------------------- super-block GEMV kernel

struct GemvKArgs {
  const uint8_t* w;
  int sbb;
  int stages;  // ring depth per warp (2..4)
  int ntiles, nchunks, gc, ngroups;
  long long nsb;
  int k;
  const float* x;
  int ldx;
  int rows;
  const float* norm_w;
  float eps;
  float* ws;
  int* counters;
  DeviceStatus* status;
  EpiParams epi;
};

struct GemvSmem {
  size_t ring, bars, frag, side, parts, red, misc, total;
};

template <int QT, int M>
__host__ __device__ GemvSmem gemv_smem_layout(int gc, int nslots, int sbb, int stages) {
  GemvSmem s;
  s.ring = (size_t)kGemvWarps * stages * sbb;
  s.bars = (size_t)kGemvWarps * kMaxStages * 8;
  s.frag = (size_t)nslots * gc * frag_chunk_u32<M>() * 4;
  s.side = (size_t)nslots * gc * side_per_chunk<QT, M>() * 4;
  s.parts = (size_t)win_sbs<M>() * 16 * M * 4;
  s.red = (size_t)kGemvWarps * (16 * M + kSegList) * 4;
  s.misc = 256 + (size_t)(kWinRuns + 1) * 4 + (size_t)kWinRuns * 12;
  s.total = s.ring + s.bars + s.frag + s.side + s.parts + s.red + s.misc;
  return s;
}

// Lane 0's side of a warp's weight ring for one matrix: the warp's remaining
// super-blocks cb + warp, cb + warp + 16, ... as a pointer walk.
struct LinearRefill {
  const uint8_t* next;
  long long step;  // 16 super-blocks, in bytes
  int left, sbb;
  int inflight;    // copies issued and not yet consumed
  uint8_t* ring;
  uint64_t* bars;
  __device__ __forceinline__ void operator()(int slot) {
    if (left <= 0) return;
    mbar_arrive_expect_tx(bars + slot, sbb);
    bulk_g2s(ring + (size_t)slot * sbb, next, sbb, bars + slot);
    next += step;
    --left;
    ++inflight;
  }
};

template <int QT, int M, bool NORM>
__global__ void __launch_bounds__(kGemvWarps * 32, 1) gemv_sb_kernel(const GemvKArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sbb = a.sbb, S = a.stages;
  const int nslots = a.ngroups > 1 ? 2 : 1;
  const GemvSmem L = gemv_smem_layout<QT, M>(a.gc, nslots, sbb, S);
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.ring);
  uint32_t* frag = reinterpret_cast<uint32_t*>(smem + L.ring + L.bars);
  float* side = reinterpret_cast<float*>(smem + L.ring + L.bars + L.frag);
  float* parts = reinterpret_cast<float*>(smem + L.ring + L.bars + L.frag + L.side);
  float* red = parts + L.parts / 4;
  uint8_t* misc = reinterpret_cast<uint8_t*>(red + L.red / 4);
  float* inv_rms = reinterpret_cast<float*>(misc);            // [M]
  float* part = inv_rms + 4;                                   // [kGemvWarps]
  int* nruns_s = reinterpret_cast<int*>(part + kGemvWarps);    // [1]
  int* ok_s = nruns_s + 1;                                     // [1]
  RunTable rt;
  rt.u0 = reinterpret_cast<int*>(misc + 256);                  // [kWinRuns + 1]
  rt.t = reinterpret_cast<int*>(rt.u0 + kWinRuns + 1);         // [kWinRuns]
  rt.grp = rt.t + kWinRuns;
  rt.cc0 = rt.grp + kWinRuns;

  const int G = gridDim.x;
  const int cb = cta_start(blockIdx.x, G, a.ntiles, a.nchunks, a.gc, a.ngroups);
  const int ce = cta_start(blockIdx.x + 1, G, a.ntiles, a.nchunks, a.gc, a.ngroups);
  uint64_t* mybars = bars + warp * kMaxStages;
  uint8_t* myring = ring + (size_t)warp * S * sbb;

  // 1. Barriers, then start streaming weights (independent of the previous
  //    kernel): warp w takes super-blocks cb + w, cb + w + 16, ...
  LinearRefill refill;
  refill.next = a.w + (size_t)(cb + warp) * sbb;
  refill.step = (long long)kGemvWarps * sbb;
  refill.left = cb + warp < ce ? (ce - cb - warp + kGemvWarps - 1) / kGemvWarps : 0;
  refill.sbb = sbb;
  refill.inflight = 0;
  refill.ring = myring;
  refill.bars = mybars;
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&mybars[s], 1);
    fence_mbar_init();
    fence_proxy_async_smem();
    for (int s = 0; s < S; ++s) refill(s);
  }
  __syncwarp();
  // The next kernel may be scheduled as soon as an SM has room; it waits for
  // this grid to complete before reading anything this grid writes.
  pdl_launch_dependents();
  // 2. Inputs of the previous kernel are visible after this.
  pdl_wait();
  if (cb >= ce) return;  // block-uniform; no copies were issued
  const int g0 = sb_decode(cb, a.ntiles, a.nchunks, a.gc).grp;
  const int g1 = sb_decode(ce - 1, a.ntiles, a.nchunks, a.gc).grp;

  // 3. Stage x (normalised if fused) for the <= 2 chunk groups this CTA touches.
  if (M == 1) {
    stage_x_m1<QT>(a.x, a.k, NORM ? a.norm_w : nullptr, a.eps, a.gc, a.nchunks, g0, g1, frag,
                   side, part, inv_rms);
  } else {
    if (NORM) norm_inv_rms(a.x, a.ldx, a.rows, a.k, a.eps, part, inv_rms);
    stage_x<QT, M>(a.x, a.ldx, a.rows, a.k, NORM ? a.norm_w : nullptr, inv_rms, a.gc, a.nchunks,
                   g0, g1, frag, side);
  }

  // 4. Windows of the range: stream, then finish their runs.
  const FinishGeom fg{a.ntiles, a.nchunks, a.gc, a.ngroups, a.rows};
  int slot = 0;
  uint32_t parity = 0;
  if (threadIdx.x == 0) *ok_s = 1;
  for (int wb = cb; wb < ce;) {
    build_window_par(wb, ce, a.ntiles, a.nchunks, a.gc, a.ngroups, kWinRuns, win_sbs<M>(), rt,
                     nruns_s);
    __syncthreads();  // run table (and the staged x) visible; parts free
    const int nruns = *nruns_s;
    const int we = rt.u0[nruns];
    if (!consume_window<QT, M>(cb, wb, we, a.ntiles, a.nchunks, a.gc, g0, frag, side, parts,
                               myring, mybars, sbb, S, slot, parity, refill.inflight, a.status,
                               2, refill))
      *ok_s = 0;  // every writer stores 0
    __syncthreads();
    if (!*ok_s) {  // a bounded wait gave up (status recorded): leave together
      if (lane == 0) ring_drain(mybars, S, slot, parity, refill.inflight);
      return;
    }
    finish_runs<M>(parts, red, rt, nruns, wb, fg, a.ws, a.counters, a.epi);
    __syncthreads();
    wb = we;
  }
}

// ------------------------------------------------------------ F32 GEMV kernel
// Warp per 16-row tile over the full K (tied F32 lm_head, F32 models).
template <int M, bool NORM>
__global__ void __launch_bounds__(256) gemv_f32_kernel(const float* w, int ntiles, int k,
                                                       const float* x, int ldx, int rows,
                                                       const float* norm_w, float eps,
                                                       EpiParams epi) {
  __shared__ float red[8][16 * M];
  __shared__ float inv[M];
  __shared__ float part[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  if (NORM) {
    for (int r = 0; r < rows; ++r) {
      float ss = 0.0f;
      for (int i = threadIdx.x; i < k; i += blockDim.x) ss = fmaf(x[(size_t)r * ldx + i], x[(size_t)r * ldx + i], ss);
      ss = warp_sum(ss);
      if (lane == 0) part[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < 8; ++i) t += part[i];
        inv[r] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)k), eps)));
      }
      __syncthreads();
    }
  }
  pdl_launch_dependents();
  for (int t = blockIdx.x * 8 + warp; t < ntiles; t += gridDim.x * 8) {
    float acc[16][M];
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int r = 0; r < M; ++r) acc[i][r] = 0.0f;
    for (int kk = lane; kk < k; kk += 32) {
      float xv[M];
#pragma unroll
      for (int r = 0; r < M; ++r) {
        xv[r] = r < rows ? x[(size_t)r * ldx + kk] : 0.0f;
        if (NORM && r < rows) xv[r] = __fmul_rn(__fmul_rn(xv[r], inv[r]), norm_w[kk]);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float wv = w[((size_t)t * 16 + i) * k + kk];
#pragma unroll
        for (int r = 0; r < M; ++r) acc[i][r] = fmaf(wv, xv[r], acc[i][r]);
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int r = 0; r < M; ++r) {
        float s = warp_sum(acc[i][r]);
        if (lane == 0) red[warp][i * M + r] = s;
      }
    __syncwarp();
    for (int i = lane; i < 16 * M; i += 32) {
      int row = i / M, r = i - row * M;
      if (r < rows) epilogue_row<M>(epi, t, row, r, red[warp]);
    }
    if (epi.argmax_key) {
      unsigned long long key = 0ull;
      if (lane < 16 && t * 16 + lane < epi.n_out)
        key = argmax_key_of(red[warp][lane * M], epi.argmax_base + t * 16 + lane);
      key = warp_max_u64(key);
      if (lane == 0 && key) atomicMax(epi.argmax_key, key);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------ launcher

static int pick_batch(int rows) { return rows <= 1 ? 1 : (rows == 2 ? 2 : 4); }

// Largest number of chunk groups any CTA range touches when the group-tiles
// are split over G CTAs.
static int cta_groups(const QMatrix& m, int G) {
  int worst = 0;
  for (int c = 0; c < G; ++c) {
    const int u = cta_start(c, G, m.ntiles, m.nchunks, m.gc, m.ngroups);
    const int ce = cta_start(c + 1, G, m.ntiles, m.nchunks, m.gc, m.ngroups);
    if (u >= ce) continue;
    const int g0 = sb_decode(u, m.ntiles, m.nchunks, m.gc).grp;
    const int g1 = sb_decode(ce - 1, m.ntiles, m.nchunks, m.gc).grp;
    worst = std::max(worst, g1 - g0 + 1);
  }
  return worst;
}

// Grid for a matrix: one CTA per SM (at most one per group-tile), more when a
// CTA range would touch more chunk groups than its staged activations hold.
template <int M>
static long long choose_grid(const QMatrix& m, int sms) {
  const int idx = M == 1 ? 0 : (M == 2 ? 1 : 2);
  if (m.grid_cache[idx] > 0) return m.grid_cache[idx];
  const long long ngt = (long long)m.ngroups * m.ntiles;
  long long G = std::min<long long>(sms, ngt);
  while (G < ngt && cta_groups(m, (int)G) > 2) G = std::min<long long>(ngt, G + sms);
  m.grid_cache[idx] = (int)G;
  return G;
}

template <int QT, int M, bool NORM>
static void launch_sb(const QMatrix& m, const float* x, int rows, int ldx, const NormSpec& norm,
                      const EpiParams& epi, const GemvWorkspace& ws, cudaStream_t stream,
                      bool pdl, int grid_ctas) {
  int dev = 0;
  MLB_CUDA(cudaGetDevice(&dev));
  const int sbb = sb_bytes(QT);
  const int nslots = m.ngroups > 1 ? 2 : 1;
  constexpr size_t kSmemMax = 227 * 1024;
  const size_t fixed = gemv_smem_layout<QT, M>(m.gc, nslots, sbb, 0).total;
  const int stages = (int)std::min<size_t>(
      kRingStages, fixed < kSmemMax ? (kSmemMax - fixed) / ((size_t)kGemvWarps * sbb) : 0);
  if (stages < 1) invalid("gemv: staged activations leave no room for the weight ring");
  const size_t smem = gemv_smem_layout<QT, M>(m.gc, nslots, sbb, stages).total;
  static size_t smem_set[64] = {};
  if (dev < 64 && smem_set[dev] < smem) {
    MLB_CUDA(cudaFuncSetAttribute(gemv_sb_kernel<QT, M, NORM>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set[dev] = smem;
  }
  const long long grid = grid_ctas > 0 ? grid_ctas : choose_grid<M>(m, sm_count(dev));
  if ((size_t)m.ntiles * m.nchunks * 16 * M > ws.partial_floats || (size_t)m.ntiles > ws.counter_count)
    invalid("gemv: workspace too small");
  GemvKArgs a;
  a.w = m.data;
  a.sbb = sbb;
  a.stages = stages;
  a.ntiles = m.ntiles;
  a.nchunks = m.nchunks;
  a.gc = m.gc;
  a.ngroups = m.ngroups;
  a.nsb = m.nsb;
  a.k = m.k;
  a.x = x;
  a.ldx = ldx;
  a.rows = rows;
  a.norm_w = norm.weight;
  a.eps = norm.eps;
  a.ws = ws.partials;
  a.counters = ws.counters;
  a.status = ws.status;
  a.epi = epi;
  launch_pdl(gemv_sb_kernel<QT, M, NORM>, dim3((unsigned)grid), dim3(kGemvWarps * 32), smem,
             stream, pdl, a);
}

template <int QT, int M>
static void dispatch_norm(const QMatrix& m, const float* x, int rows, int ldx,
                          const NormSpec& norm, const EpiParams& epi, const GemvWorkspace& ws,
                          cudaStream_t stream, bool pdl, int grid) {
  if (norm.weight)
    launch_sb<QT, M, true>(m, x, rows, ldx, norm, epi, ws, stream, pdl, grid);
  else
    launch_sb<QT, M, false>(m, x, rows, ldx, norm, epi, ws, stream, pdl, grid);
}

template <int QT>
static void dispatch_m(int mb, const QMatrix& m, const float* x, int rows, int ldx,
                       const NormSpec& norm, const EpiParams& epi, const GemvWorkspace& ws,
                       cudaStream_t stream, bool pdl, int grid) {
  if (mb == 1)
    dispatch_norm<QT, 1>(m, x, rows, ldx, norm, epi, ws, stream, pdl, grid);
  else if (mb == 2)
    dispatch_norm<QT, 2>(m, x, rows, ldx, norm, epi, ws, stream, pdl, grid);
  else
    dispatch_norm<QT, 4>(m, x, rows, ldx, norm, epi, ws, stream, pdl, grid);
}

template <int M>
static void launch_f32(const QMatrix& m, const float* x, int rows, int ldx, const NormSpec& norm,
                       const EpiParams& epi, cudaStream_t stream, bool pdl) {
  int dev = 0;
  MLB_CUDA(cudaGetDevice(&dev));
  int grid = std::max(1, std::min((m.ntiles + 7) / 8, sm_count(dev) * 4));
  if (norm.weight)
    launch_pdl(gemv_f32_kernel<M, true>, dim3(grid), dim3(256), 0, stream, pdl,
               reinterpret_cast<const float*>(m.data), m.ntiles, m.k, x, ldx, rows, norm.weight,
               norm.eps, epi);
  else
    launch_pdl(gemv_f32_kernel<M, false>, dim3(grid), dim3(256), 0, stream, pdl,
               reinterpret_cast<const float*>(m.data), m.ntiles, m.k, x, ldx, rows, norm.weight,
               norm.eps, epi);
}

int gemv_kernel_count(const QMatrix& m, int rows) {
  (void)m;
  return (rows + kMaxBatch - 1) / kMaxBatch;
}

void gemv_launch(const QMatrix& m, const float* x, int rows, int ldx, const NormSpec& norm,
                 const EpiParams& epi_in, const GemvWorkspace& ws, cudaStream_t stream, bool pdl,
                 int grid_ctas) {
  if (rows < 1) invalid("gemv: rows must be positive");
  for (int r0 = 0; r0 < rows; r0 += kMaxBatch) {
    int nr = std::min(kMaxBatch, rows - r0);
    EpiParams epi = epi_in;
    epi.y = epi_in.y ? epi_in.y + (size_t)r0 * epi_in.ldy : nullptr;
    epi.resid = epi_in.resid ? epi_in.resid + (size_t)r0 * epi_in.ldr : nullptr;
    if (epi.kind == kEpiQkv && rows > 1) invalid("gemv: fused QKV epilogue takes one row");
    const float* xr = x + (size_t)r0 * ldx;
    int mb = pick_batch(nr);
    bool p = pdl && r0 == 0;
    if (m.qtype == MLB_F32) {
      if (mb == 1) launch_f32<1>(m, xr, nr, ldx, norm, epi, stream, p);
      else if (mb == 2) launch_f32<2>(m, xr, nr, ldx, norm, epi, stream, p);
      else launch_f32<4>(m, xr, nr, ldx, norm, epi, stream, p);
    } else if (m.qtype == MLB_Q4_0) {
      dispatch_m<MLB_Q4_0>(mb, m, xr, nr, ldx, norm, epi, ws, stream, p, grid_ctas);
    } else if (m.qtype == MLB_Q4_1) {
      dispatch_m<MLB_Q4_1>(mb, m, xr, nr, ldx, norm, epi, ws, stream, p, grid_ctas);
    } else {
      dispatch_m<MLB_Q8_0>(mb, m, xr, nr, ldx, norm, epi, ws, stream, p, grid_ctas);
    }
  }
}

// ---------------------------------------------- generic GEMV over raw blocks
// One warp per (output row, batch row); lanes stride over the GGUF blocks of
// the row. Used by the standalone entry points, which take raw GGUF pointers.
template <int QT>
__global__ void gemv_gguf_kernel(const float* __restrict__ x, int rows, int k,
                                 const uint8_t* __restrict__ w, int n, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= (long long)n * rows) return;
  const int j = (int)(wid % n), r = (int)(wid / n);
  const float* xr = x + (size_t)r * k;
  float acc = 0.0f;
  if (QT == MLB_F32) {
    const float* wr = reinterpret_cast<const float*>(w) + (size_t)j * k;
    for (int kk = lane; kk < k; kk += 32) acc = fmaf(wr[kk], xr[kk], acc);
  } else {
    const int nb = (k + 31) / 32;
    const int bsz = QT == MLB_Q8_0 ? 34 : (QT == MLB_Q4_1 ? 20 : 18);
    const uint8_t* wr = w + (size_t)j * nb * bsz;
    for (int b = lane; b < nb; b += 32) {
      const uint8_t* blk = wr + (size_t)b * bsz;
      const uint16_t dbits = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
      const float d = __half2float(__ushort_as_half(dbits));
      float m = 0.0f;
      if (QT == MLB_Q4_1)
        m = __half2float(__ushort_as_half((uint16_t)blk[2] | ((uint16_t)blk[3] << 8)));
      const int kend = min(32, k - b * 32);
      float s = 0.0f, sx = 0.0f;
      for (int i = 0; i < kend; ++i) {
        float xv = xr[b * 32 + i];
        float q;
        if (QT == MLB_Q8_0) {
          q = (float)(int8_t)blk[2 + i];
        } else {
          const uint8_t byte = blk[(QT == MLB_Q4_1 ? 4 : 2) + (i & 15)];
          int nib = i < 16 ? (byte & 15) : (byte >> 4);
          q = (float)(QT == MLB_Q4_0 ? nib - 8 : nib);
        }
        s = fmaf(q, xv, s);
        sx += xv;
      }
      acc = fmaf(d, s, acc);
      if (QT == MLB_Q4_1) acc = fmaf(m, sx, acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) y[(size_t)r * n + j] = acc;
}

void gemv_gguf(int qtype, const float* x, int rows, int k, const void* w, int n, float* y,
               cudaStream_t stream) {
  long long warps = (long long)n * rows;
  unsigned grid = (unsigned)((warps * 32 + 255) / 256);
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  switch (qtype) {
    case MLB_F32: gemv_gguf_kernel<MLB_F32><<<grid, 256, 0, stream>>>(x, rows, k, wb, n, y); break;
    case MLB_Q8_0: gemv_gguf_kernel<MLB_Q8_0><<<grid, 256, 0, stream>>>(x, rows, k, wb, n, y); break;
    case MLB_Q4_0: gemv_gguf_kernel<MLB_Q4_0><<<grid, 256, 0, stream>>>(x, rows, k, wb, n, y); break;
    case MLB_Q4_1: gemv_gguf_kernel<MLB_Q4_1><<<grid, 256, 0, stream>>>(x, rows, k, wb, n, y); break;
    default: invalid("linear: unsupported quant type " + std::to_string(qtype));
  }
  MLB_CUDA(cudaGetLastError());
}

}  // namespace mlb

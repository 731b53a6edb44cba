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
  int mb = max_batch < 1 ? 1 : (max_batch > kMaxBatch ? kMaxBatch : max_batch);
  int gc = 16 / (mb >= 3 ? 4 : mb);
  m.gc = std::min(gc, m.nchunks);
  m.ngroups = (m.nchunks + m.gc - 1) / m.gc;
  m.nsb = (long long)m.ntiles * m.nchunks;
  m.bytes = (size_t)m.nsb * sb_bytes(qtype);
}

__host__ __device__ inline long long sb_index(int t, int c, int ntiles, int nchunks, int gc) {
  int grp = c / gc;
  int cc = c - grp * gc;
  int geff = min(gc, nchunks - grp * gc);
  return (long long)grp * ntiles * gc + (long long)t * geff + cc;
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

// --------------------------------------------------------------- epilogues

template <int M>
__device__ void epilogue_row(const EpiParams& p, int tile, int row, int r, const float* vals) {
  float v = vals[row * M + r];
  int grow = tile * 16 + row;
  switch (p.kind) {
    case kEpiStore:
      if (grow < p.n_out) p.y[(size_t)r * p.ldy + grow] = v;
      break;
    case kEpiResidual:
      if (grow < p.n_out)
        p.y[(size_t)r * p.ldy + grow] = __fadd_rn(p.resid[(size_t)r * p.ldr + grow], v);
      break;
    case kEpiSwiglu: {
      if (row >= 8) break;
      int h = tile * 8 + row;
      if (h >= p.n_out) break;
      float g = v, u = vals[(row + 8) * M + r];
      float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
      p.y[(size_t)r * p.ldy + h] = __fmul_rn(__fmul_rn(g, sg), u);
      break;
    }
    case kEpiQkv: {
      int local, size, sec;
      if (grow < p.k_off) {
        sec = 0; local = grow; size = p.q_rows;
      } else if (grow < p.v_off) {
        sec = 1; local = grow - p.k_off; size = p.kv_rows;
      } else {
        sec = 2; local = grow - p.v_off; size = p.kv_rows;
      }
      if (local >= size) break;
      const int D = p.head_dim;
      auto logical = [&](int l) {
        if (!p.neox || sec == 2) return l;
        int hd = l / D, q = l - hd * D;
        return hd * D + ((q & 1) ? (q >> 1) + D / 2 : (q >> 1));
      };
      const int bias_base = sec == 0 ? 0 : (sec == 1 ? p.q_rows : p.q_rows + p.kv_rows);
      int L = logical(local);
      if (p.bias) v = __fadd_rn(v, p.bias[bias_base + L]);
      int pos = *p.pos;
      if (sec == 2) {
        p.values[(size_t)pos * p.kv_rows + L] = v;
        break;
      }
      int partner = local ^ 1;
      float w = vals[(row ^ 1) * M + r];
      if (p.bias) w = __fadd_rn(w, p.bias[bias_base + logical(partner)]);
      int in_head = L % D;
      int j;
      bool first;
      if (p.neox) {
        first = in_head < D / 2;
        j = first ? in_head : in_head - D / 2;
      } else {
        first = (in_head & 1) == 0;
        j = in_head >> 1;
      }
      float2 cs = p.rope[(size_t)pos * (D / 2) + j];
      float out;
      if (first)  // a*c - b*s with a = this, b = partner (src/ops.cc:155, 174)
        out = __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(w, cs.y));
      else        // a*s + b*c with a = partner, b = this (src/ops.cc:156, 175)
        out = __fadd_rn(__fmul_rn(w, cs.y), __fmul_rn(v, cs.x));
      if (sec == 0)
        p.q_out[(size_t)r * p.q_rows + L] = out;
      else
        p.keys[(size_t)pos * p.kv_rows + L] = out;
      break;
    }
  }
}

// ---------------------------------------------------- super-block GEMV kernel

struct GemvKArgs {
  const uint8_t* w;
  int sbb;
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

struct SbPos {
  int grp, t, cc, geff;
};

__device__ __forceinline__ SbPos sb_decode(long long u, int ntiles, int nchunks, int gc) {
  SbPos s;
  long long per = (long long)ntiles * gc;
  s.grp = (int)(u / per);
  long long rem = u - (long long)s.grp * per;
  s.geff = min(gc, nchunks - s.grp * gc);
  s.t = (int)(rem / s.geff);
  s.cc = (int)(rem - (long long)s.t * s.geff);
  return s;
}

__device__ __forceinline__ long long warp_start(long long w, long long nsb, long long W) {
  return nsb * w / W;
}

// Calls f(start_chunk) for every segment tile t is split into by the static
// partition (chunk-group runs cut at warp-range boundaries), in chunk order.
// Works for any warp count, including warps with empty ranges.
template <class F>
__device__ __forceinline__ int for_each_segment(int t, int ntiles, int nchunks, int gc,
                                                int ngroups, long long nsb, long long W, F f) {
  int n = 0;
  for (int gr = 0; gr < ngroups; ++gr) {
    const int geff = min(gc, nchunks - gr * gc);
    const long long u0 = (long long)gr * ntiles * gc + (long long)t * geff, end = u0 + geff;
    long long p = u0;
    while (p < end) {
      const long long w = ((p + 1) * W + nsb - 1) / nsb - 1;  // warp whose range holds p
      const long long e = warp_start(w + 1, nsb, W);
      f(gr * gc + (int)(p - u0));
      ++n;
      p = e < end ? e : end;
    }
  }
  return n;
}

constexpr int kFragLaneStride = 36;  // u32 per lane per chunk (32 + 4 pad: no bank conflicts)

template <int M>
__host__ __device__ constexpr int frag_chunk_u32() {
  return 8 * M * kFragLaneStride;
}

template <int QT, int M>
__host__ __device__ constexpr int red_floats() {
  return kGemvWarps * 16 * M;
}

template <int QT, int M>
size_t gemv_smem_bytes(int gc, int sbb) {
  size_t ring = (size_t)kGemvWarps * kGemvStages * sbb;
  size_t bars = (size_t)kGemvWarps * kGemvStages * 8;
  size_t frag = (size_t)2 * gc * frag_chunk_u32<M>() * 4;
  size_t bsum = QT == MLB_Q4_1 ? (size_t)2 * gc * 8 * M * 4 : 0;
  size_t red = (size_t)red_floats<QT, M>() * 4;
  return ring + bars + frag + bsum + red + 64;
}

template <int QT, int M, bool NORM>
__global__ void __launch_bounds__(kGemvWarps * 32, 1) gemv_sb_kernel(const GemvKArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sbb = a.sbb;
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + (size_t)kGemvWarps * kGemvStages * sbb);
  uint32_t* frag = reinterpret_cast<uint32_t*>(bars + kGemvWarps * kGemvStages);
  const int slot_u32 = a.gc * frag_chunk_u32<M>();
  float* bsum = reinterpret_cast<float*>(frag + 2 * slot_u32);
  const int bsum_slot = a.gc * 8 * M;
  float* red = bsum + (QT == MLB_Q4_1 ? 2 * bsum_slot : 0);
  float* misc = red + red_floats<QT, M>();  // inv_rms[M], partial sums

  const long long W = (long long)gridDim.x * kGemvWarps;
  const long long wg = (long long)blockIdx.x * kGemvWarps + warp;
  const long long ub = warp_start(wg, a.nsb, W), ue = warp_start(wg + 1, a.nsb, W);
  const long long cb = warp_start((long long)blockIdx.x * kGemvWarps, a.nsb, W);
  const long long ce = warp_start((long long)(blockIdx.x + 1) * kGemvWarps, a.nsb, W);
  uint64_t* mybars = bars + warp * kGemvStages;
  uint8_t* myring = ring + (size_t)warp * kGemvStages * sbb;

  // 1. Barriers, then start streaming weights (independent of the previous kernel).
  if (lane == 0) {
    for (int s = 0; s < kGemvStages; ++s) mbar_init(&mybars[s], 1);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  __syncwarp();
  if (lane == 0) {
    for (int s = 0; s < kGemvStages && ub + s < ue; ++s) {
      mbar_arrive_expect_tx(&mybars[s], sbb);
      bulk_g2s(myring + (size_t)s * sbb, a.w + (size_t)(ub + s) * sbb, sbb, &mybars[s]);
    }
  }

  // 2. Inputs of the previous kernel are visible after this.
  pdl_wait();

  const int rows = a.rows;
  if (NORM) {
    // inv_rms[r] = 1 / sqrt(sum(x^2)/K + eps), src/ops.cc:55-61 (tree order).
    float* part = misc + M;
    for (int r = 0; r < rows; ++r) {
      float ss = 0.0f;
      const float* xr = a.x + (size_t)r * a.ldx;
      for (int i = threadIdx.x; i < a.k; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
      ss = warp_sum(ss);
      if (lane == 0) part[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < kGemvWarps; ++w) t += part[w];
        t = __fdiv_rn(t, (float)a.k);
        misc[r] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(t, a.eps)));
      }
      __syncthreads();
    }
  }

  // 3. Stage x (normalised if fused) for the <= 2 chunk groups this CTA touches,
  //    in mma B-fragment order, split into fp16 hi + lo.
  int g0 = 0, g1 = -1;
  if (ce > cb) {
    g0 = sb_decode(cb, a.ntiles, a.nchunks, a.gc).grp;
    g1 = sb_decode(ce - 1, a.ntiles, a.nchunks, a.gc).grp;
  }
  if (g1 - g0 > 1) {  // host guarantees <= 2 groups per CTA
    if (threadIdx.x == 0 && a.status) {
      atomicExch(&a.status->code, MLB_ERR_INVALID);
      atomicExch(&a.status->where, 1);
    }
    return;
  }
  for (int j = 0; j <= g1 - g0; ++j) {
    const int grp = g0 + j;
    const int geff = min(a.gc, a.nchunks - grp * a.gc);
    const int kbase = grp * a.gc * kChunkK;
    uint32_t* fs = frag + j * slot_u32;
    const int pairs = geff * 128 * M;
    for (int idx = threadIdx.x; idx < pairs; idx += blockDim.x) {
      int r = idx / (geff * 128);
      int rem = idx - r * geff * 128;
      int cc = rem >> 7, pe = rem & 127;
      int kk = pe * 2;
      int s = kk >> 4, wv = kk & 15;
      int reg = wv >= 8, cl = (wv & 7) >> 1;
      int k = kbase + cc * kChunkK + kk;
      float x0 = 0.0f, x1 = 0.0f;
      if (r < rows) {
        const float* xr = a.x + (size_t)r * a.ldx;
        if (k < a.k) x0 = xr[k];
        if (k + 1 < a.k) x1 = xr[k + 1];
        if (NORM) {
          float sc = misc[r];
          if (k < a.k) x0 = __fmul_rn(__fmul_rn(x0, sc), a.norm_w[k]);
          if (k + 1 < a.k) x1 = __fmul_rn(__fmul_rn(x1, sc), a.norm_w[k + 1]);
        }
      }
      __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
      __half l0 = __float2half_rn(x0 - __half2float(h0));
      __half l1 = __float2half_rn(x1 - __half2float(h1));
      uint32_t* base = fs + cc * frag_chunk_u32<M>();
      int lane_hi = 4 * (2 * r) + cl, lane_lo = lane_hi + 4;
      base[lane_hi * kFragLaneStride + s * 2 + reg] = h2_as_u32(__halves2half2(h0, h1));
      base[lane_lo * kFragLaneStride + s * 2 + reg] = h2_as_u32(__halves2half2(l0, l1));
    }
    if (QT == MLB_Q4_1) {
      float* bs = bsum + j * bsum_slot;
      for (int idx = threadIdx.x; idx < geff * 8 * M; idx += blockDim.x) {
        int r = idx % M, b = (idx / M) & 7, cc = idx / (8 * M);
        float s = 0.0f;
        int k0 = kbase + cc * kChunkK + b * 32;
        if (r < rows) {
          const float* xr = a.x + (size_t)r * a.ldx;
          for (int i = 0; i < 32 && k0 + i < a.k; ++i) {
            float xv = xr[k0 + i];
            if (NORM) xv = __fmul_rn(__fmul_rn(xv, misc[r]), a.norm_w[k0 + i]);
            s += xv;
          }
        }
        bs[(cc * 8 + b) * M + r] = s;
      }
    }
  }
  __syncthreads();
  // Let the next kernel launch and begin its own weight prefetch.
  pdl_launch_dependents();

  // 4. Stream this warp's super-blocks.
  const int g = lane >> 2, cl = lane & 3;
  const bool bl = lane < 8 * M;  // lanes carrying B-fragment columns
  float* myred = red + warp * 16 * M;
  float acc0 = 0.0f, acc1 = 0.0f;
  int cur_t = -1, cur_grp = -1, seg_c0 = 0;
  int b_chunk = -1;
  uint32_t B[16][2];
#pragma unroll
  for (int s = 0; s < 16; ++s) B[s][0] = B[s][1] = 0u;

  auto flush = [&](int t, int grp, int c0) {
    // Per-lane accumulators -> myred[row][r]
    __syncwarp();
    if (cl < M) {
      myred[g * M + cl] = acc0;
      myred[(g + 8) * M + cl] = acc1;
    }
    __syncwarp();
    // Number of segments tile t is split into (static partition).
    const int nseg = for_each_segment(t, a.ntiles, a.nchunks, a.gc, a.ngroups, a.nsb, W,
                                      [](int) {});
    bool finish = true;
    if (nseg > 1) {
      float* slot = a.ws + ((size_t)t * a.nchunks + c0) * 16 * M;
      for (int i = lane; i < 16 * M; i += 32) slot[i] = myred[i];
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = (atomicAdd(&a.counters[t], 1) == nseg - 1);
      last = __shfl_sync(0xffffffffu, last, 0);
      finish = last != 0;
      if (finish) {
        __threadfence();
        // Sum every segment of the tile in chunk order (deterministic).
        for (int i = lane; i < 16 * M; i += 32) {
          float s = 0.0f;
          for_each_segment(t, a.ntiles, a.nchunks, a.gc, a.ngroups, a.nsb, W, [&](int c) {
            s += __ldcg(a.ws + ((size_t)t * a.nchunks + c) * 16 * M + i);
          });
          myred[i] = s;
        }
        if (lane == 0) a.counters[t] = 0;
        __syncwarp();
      }
    }
    if (finish) {
      for (int i = lane; i < 16 * M; i += 32) {
        int row = i / M, r = i - row * M;
        if (r < rows) epilogue_row<M>(a.epi, t, row, r, myred);
      }
    }
    __syncwarp();
    acc0 = 0.0f;
    acc1 = 0.0f;
  };

  long long it = 0;
  for (long long u = ub; u < ue; ++u, ++it) {
    const SbPos sp = sb_decode(u, a.ntiles, a.nchunks, a.gc);
    if (sp.t != cur_t || sp.grp != cur_grp) {
      if (cur_t >= 0) flush(cur_t, cur_grp, seg_c0);
      cur_t = sp.t;
      cur_grp = sp.grp;
      seg_c0 = sp.grp * a.gc + sp.cc;
    }
    const int chunk = sp.grp * a.gc + sp.cc;
    if (chunk != b_chunk) {
      b_chunk = chunk;
      if (bl) {
        const uint32_t* fsrc =
            frag + (sp.grp - g0) * slot_u32 + sp.cc * frag_chunk_u32<M>() + lane * kFragLaneStride;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          uint4 v = *reinterpret_cast<const uint4*>(fsrc + s * 4);
          B[2 * s][0] = v.x;
          B[2 * s][1] = v.y;
          B[2 * s + 1][0] = v.z;
          B[2 * s + 1][1] = v.w;
        }
      }
    }
    const int slot = (int)(it % kGemvStages);
    const uint32_t parity = (uint32_t)((it / kGemvStages) & 1);
    if (!mbar_wait_bounded(&mybars[slot], parity, a.status, 2)) return;
    const uint8_t* sb = myring + (size_t)slot * sbb;

    const int qbytes = QT == MLB_Q8_0 ? 4096 : 2048;
    const uint4 sc0 = *reinterpret_cast<const uint4*>(sb + qbytes + g * 32);
    const uint4 sc1 = *reinterpret_cast<const uint4*>(sb + qbytes + g * 32 + 16);
    const uint32_t scw[8] = {sc0.x, sc0.y, sc0.z, sc0.w, sc1.x, sc1.y, sc1.z, sc1.w};
    uint32_t mnw[8];
    if (QT == MLB_Q4_1) {
      const uint4 m0 = *reinterpret_cast<const uint4*>(sb + 2304 + g * 32);
      const uint4 m1 = *reinterpret_cast<const uint4*>(sb + 2304 + g * 32 + 16);
      mnw[0] = m0.x; mnw[1] = m0.y; mnw[2] = m0.z; mnw[3] = m0.w;
      mnw[4] = m1.x; mnw[5] = m1.y; mnw[6] = m1.z; mnw[7] = m1.w;
    }

#pragma unroll
    for (int b = 0; b < 8; ++b) {
      uint32_t A1[4], A2[4];
      if (QT == MLB_Q8_0) {
        const uint4 q = *reinterpret_cast<const uint4*>(sb + (size_t)(b * 32 + lane) * 16);
        const __half2 bias = __float2half2_rn(1152.0f);
        const uint32_t wx[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                                q.w ^ 0x80808080u};
        // wx[0]: row g (k 2c,2c+1,2c+8,2c+9), wx[1]: row g (+16), wx[2..3]: row g+8
        A1[0] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[0], 0x64646464u, 0x4140)), bias));
        A1[2] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[0], 0x64646464u, 0x4342)), bias));
        A1[1] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[2], 0x64646464u, 0x4140)), bias));
        A1[3] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[2], 0x64646464u, 0x4342)), bias));
        A2[0] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[1], 0x64646464u, 0x4140)), bias));
        A2[2] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[1], 0x64646464u, 0x4342)), bias));
        A2[1] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[3], 0x64646464u, 0x4140)), bias));
        A2[3] = h2_as_u32(__hsub2(u32_as_h2(__byte_perm(wx[3], 0x64646464u, 0x4342)), bias));
      } else {
        const uint2 q =
            *reinterpret_cast<const uint2*>(sb + (size_t)((b >> 1) * 32 + lane) * 16 + (b & 1) * 8);
        const uint32_t w0 = q.x, w1 = q.y;  // rows g and g+8
        const uint32_t w0s = w0 >> 8, w1s = w1 >> 8;
        const uint32_t M1 = 0x000F000Fu, M2 = 0x00F000F0u, E = 0x64006400u;
        // low nibbles: 1024 + q ; high nibbles: 1024 + 16 q
        const __half2 lo_off = __float2half2_rn(QT == MLB_Q4_0 ? 1032.0f : 1024.0f);
        const __half2 hi_mul = __float2half2_rn(1.0f / 16.0f);
        const __half2 hi_off = __float2half2_rn(QT == MLB_Q4_0 ? -72.0f : -64.0f);
        A1[0] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w0, M1, E)), lo_off));
        A1[1] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w1, M1, E)), lo_off));
        A1[2] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w0s, M1, E)), lo_off));
        A1[3] = h2_as_u32(__hsub2(u32_as_h2(lop3_and_or(w1s, M1, E)), lo_off));
        A2[0] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w0, M2, E)), hi_mul, hi_off));
        A2[1] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w1, M2, E)), hi_mul, hi_off));
        A2[2] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w0s, M2, E)), hi_mul, hi_off));
        A2[3] = h2_as_u32(__hfma2(u32_as_h2(lop3_and_or(w1s, M2, E)), hi_mul, hi_off));
      }
      float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      mma_16816(d, A1, B[2 * b][0], B[2 * b][1]);
      mma_16816(d, A2, B[2 * b + 1][0], B[2 * b + 1][1]);
      const float2 sc = __half22float2(u32_as_h2(scw[b]));
      acc0 = fmaf(sc.x, d[0] + d[1], acc0);
      acc1 = fmaf(sc.y, d[2] + d[3], acc1);
      if (QT == MLB_Q4_1) {
        const float2 mn = __half22float2(u32_as_h2(mnw[b]));
        const int rr = cl < M ? cl : 0;
        const float sx = bsum[(sp.grp - g0) * bsum_slot + (sp.cc * 8 + b) * M + rr];
        acc0 = fmaf(mn.x, sx, acc0);
        acc1 = fmaf(mn.y, sx, acc1);
      }
    }
    __syncwarp();
    if (lane == 0 && u + kGemvStages < ue) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&mybars[slot], sbb);
      bulk_g2s(myring + (size_t)slot * sbb, a.w + (size_t)(u + kGemvStages) * sbb, sbb,
               &mybars[slot]);
    }
  }
  if (cur_t >= 0) flush(cur_t, cur_grp, seg_c0);
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
    __syncwarp();
  }
}

// ------------------------------------------------------------------ launcher

static int pick_batch(int rows) { return rows <= 1 ? 1 : (rows == 2 ? 2 : 4); }

template <int QT, int M, bool NORM>
static void launch_sb(const QMatrix& m, const float* x, int rows, int ldx, const NormSpec& norm,
                      const EpiParams& epi, const GemvWorkspace& ws, cudaStream_t stream,
                      bool pdl, int grid_ctas) {
  int dev = 0;
  MLB_CUDA(cudaGetDevice(&dev));
  const int sbb = sb_bytes(QT);
  const size_t smem = gemv_smem_bytes<QT, M>(m.gc, sbb);
  static size_t smem_set[64] = {};
  if (dev < 64 && smem_set[dev] < smem) {
    MLB_CUDA(cudaFuncSetAttribute(gemv_sb_kernel<QT, M, NORM>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set[dev] = smem;
  }
  int sms = sm_count(dev);
  long long grid = grid_ctas > 0 ? grid_ctas : sms;
  // Every CTA must span <= 2 chunk groups (its range must not exceed a group):
  // at least ngroups + 1 CTAs. At most one CTA per 8 super-blocks, so warps are
  // not idle; that bound alone already keeps a CTA range within 8-9 SBs, which
  // never exceeds a group of >= 16 SBs (or there is a single group).
  long long per_group = (long long)m.ntiles * m.gc;
  long long min_grid = (m.nsb + per_group - 1) / per_group + 1;
  long long max_grid = std::max(1LL, m.nsb / kGemvWarps);
  grid = std::min(std::max(grid, min_grid), max_grid);
  if ((size_t)m.ntiles * m.nchunks * 16 * M > ws.partial_floats || (size_t)m.ntiles > ws.counter_count)
    invalid("gemv: workspace too small");
  GemvKArgs a;
  a.w = m.data;
  a.sbb = sbb;
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

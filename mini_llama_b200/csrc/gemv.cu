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

struct SbPos {
  int grp, t, cc, geff;
};

__host__ __device__ inline SbPos sb_decode(long long u, int ntiles, int nchunks, int gc) {
  SbPos s;
  long long per = (long long)ntiles * gc;
  s.grp = (int)(u / per);
  long long rem = u - (long long)s.grp * per;
  s.geff = min(gc, nchunks - s.grp * gc);
  s.t = (int)(rem / s.geff);
  s.cc = (int)(rem - (long long)s.t * s.geff);
  return s;
}

// CTA c of G owns super-blocks [cta_start(c), cta_start(c + 1)).
__host__ __device__ inline long long cta_start(long long c, long long nsb, long long G) {
  return nsb * c / G;
}

// Calls f(start_chunk) for every segment tile t is split into: its runs in each
// chunk group, cut at CTA-range boundaries; in chunk order.
template <class F>
__device__ __forceinline__ int for_each_segment(int t, int ntiles, int nchunks, int gc,
                                                int ngroups, long long nsb, long long G, F f) {
  int n = 0;
  for (int gr = 0; gr < ngroups; ++gr) {
    const int geff = min(gc, nchunks - gr * gc);
    const long long u0 = (long long)gr * ntiles * gc + (long long)t * geff, end = u0 + geff;
    long long p = u0;
    while (p < end) {
      const long long c = ((p + 1) * G + nsb - 1) / nsb - 1;  // CTA whose range holds p
      const long long e = cta_start(c + 1, nsb, G);
      f(gr * gc + (int)(p - u0));
      ++n;
      p = e < end ? e : end;
    }
  }
  return n;
}

constexpr int kFragLaneStride = 36;  // u32 per lane per chunk (32 + 4 pad: no bank conflicts)
constexpr int kMaxStages = 4;
constexpr int kSegList = 32;         // segment starts gathered per pass of a fix-up

template <int M>
__host__ __device__ constexpr int frag_chunk_u32() {
  return 8 * M * kFragLaneStride;
}
// (group, tile) runs one CTA range may touch; the launcher sizes the grid so
// that no CTA exceeds it.
template <int M>
__host__ __device__ constexpr int max_cta_runs() {
  return M == 1 ? 16 : 4;
}

struct GemvSmem {
  size_t ring, bars, frag, bsum, slots, red, misc, total;
};

template <int QT, int M>
__host__ __device__ GemvSmem gemv_smem_layout(int gc, int nslots, int sbb, int stages) {
  GemvSmem s;
  s.ring = (size_t)kGemvWarps * stages * sbb;
  s.bars = (size_t)kGemvWarps * kMaxStages * 8;
  s.frag = (size_t)nslots * gc * frag_chunk_u32<M>() * 4;
  s.bsum = QT == MLB_Q4_1 ? (size_t)nslots * gc * 8 * M * 4 : 0;
  s.slots = (size_t)max_cta_runs<M>() * kGemvWarps * 16 * M * 4;
  s.red = (size_t)kGemvWarps * (16 * M + kSegList) * 4;
  s.misc = 256 + (size_t)(max_cta_runs<M>() + 1) * 8 + (size_t)max_cta_runs<M>() * 12;
  s.total = s.ring + s.bars + s.frag + s.bsum + s.slots + s.red + s.misc;
  return s;
}

template <int QT, int M, bool NORM>
__global__ void __launch_bounds__(kGemvWarps * 32, 1) gemv_sb_kernel(const GemvKArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int R = max_cta_runs<M>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sbb = a.sbb, S = a.stages;
  const int nslots = a.ngroups > 1 ? 2 : 1;
  const GemvSmem L = gemv_smem_layout<QT, M>(a.gc, nslots, sbb, S);
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.ring);
  uint32_t* frag = reinterpret_cast<uint32_t*>(smem + L.ring + L.bars);
  float* bsum = reinterpret_cast<float*>(smem + L.ring + L.bars + L.frag);
  float* slots = reinterpret_cast<float*>(smem + L.ring + L.bars + L.frag + L.bsum);
  float* red = slots + L.slots / 4;
  uint8_t* misc = reinterpret_cast<uint8_t*>(red + L.red / 4);
  float* inv_rms = reinterpret_cast<float*>(misc);            // [M]
  float* part = inv_rms + 4;                                   // [kGemvWarps]
  int* nruns_s = reinterpret_cast<int*>(part + kGemvWarps);    // [1]
  long long* run_u0 = reinterpret_cast<long long*>(misc + 256);  // [R + 1]
  int* run_t = reinterpret_cast<int*>(run_u0 + R + 1);         // [R]
  int* run_grp = run_t + R;
  int* run_cc0 = run_grp + R;
  const int slot_u32 = a.gc * frag_chunk_u32<M>();
  const int bsum_slot = a.gc * 8 * M;

  const long long G = gridDim.x;
  const long long cb = cta_start(blockIdx.x, a.nsb, G), ce = cta_start(blockIdx.x + 1, a.nsb, G);
  uint64_t* mybars = bars + warp * kMaxStages;
  uint8_t* myring = ring + (size_t)warp * S * sbb;

  // 1. Barriers, then start streaming weights (independent of the previous
  //    kernel): warp w takes super-blocks cb + w, cb + w + 16, ...
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&mybars[s], 1);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  __syncwarp();
  if (lane == 0) {
    for (int s = 0; s < S; ++s) {
      const long long u = cb + warp + (long long)s * kGemvWarps;
      if (u >= ce) break;
      mbar_arrive_expect_tx(&mybars[s], sbb);
      bulk_g2s(myring + (size_t)s * sbb, a.w + (size_t)u * sbb, sbb, &mybars[s]);
    }
  }
  // The run table of this CTA range (no dependence on the previous kernel).
  if (threadIdx.x == 0) {
    long long u = cb;
    int r = 0;
    while (u < ce && r < R) {
      const SbPos sp = sb_decode(u, a.ntiles, a.nchunks, a.gc);
      const long long len = min((long long)(sp.geff - sp.cc), ce - u);
      run_u0[r] = u;
      run_t[r] = sp.t;
      run_grp[r] = sp.grp;
      run_cc0[r] = sp.cc;
      u += len;
      ++r;
    }
    run_u0[r] = u;
    *nruns_s = (u < ce) ? -1 : r;  // -1: more runs than the launcher allowed
  }
  // The next kernel may be scheduled as soon as an SM has room; it waits for
  // this grid to complete before reading anything this grid writes.
  pdl_launch_dependents();
  // 2. Inputs of the previous kernel are visible after this.
  pdl_wait();

  const int rows = a.rows;
  if (NORM) {
    // inv_rms[r] = 1 / sqrt(sum(x^2)/K + eps), src/ops.cc:55-61 (tree order).
    for (int r = 0; r < rows; ++r) {
      float ss = 0.0f;
      const float* xr = a.x + (size_t)r * a.ldx;
      if ((a.k & 3) == 0 && (((uintptr_t)xr) & 15) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int i = threadIdx.x; i < (a.k >> 2); i += blockDim.x) {
          const float4 v = x4[i];
          ss = fmaf(v.x, v.x, ss);
          ss = fmaf(v.y, v.y, ss);
          ss = fmaf(v.z, v.z, ss);
          ss = fmaf(v.w, v.w, ss);
        }
      } else {
        for (int i = threadIdx.x; i < a.k; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) part[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < kGemvWarps; ++w) t += part[w];  // fixed order
        t = __fdiv_rn(t, (float)a.k);
        inv_rms[r] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(t, a.eps)));
      }
      __syncthreads();
    }
  } else {
    __syncthreads();  // run table visible
  }
  const int nruns = *nruns_s;
  if (nruns < 0) {
    if (threadIdx.x == 0 && a.status) {
      atomicExch(&a.status->code, MLB_ERR_INVALID);
      atomicExch(&a.status->where, 1);
    }
    return;
  }
  const int g0 = nruns > 0 ? run_grp[0] : 0;
  const int g1 = nruns > 0 ? run_grp[nruns - 1] : -1;

  // 3. Stage x (normalised if fused) for the <= 2 chunk groups this CTA touches,
  //    in mma B-fragment order, split into fp16 hi + lo; zero the run slots.
  for (int i = threadIdx.x; i < R * kGemvWarps * 16 * M; i += blockDim.x) slots[i] = 0.0f;
  for (int j = 0; j <= g1 - g0; ++j) {
    const int grp = g0 + j;
    const int geff = min(a.gc, a.nchunks - grp * a.gc);
    const int kbase = grp * a.gc * kChunkK;
    uint32_t* fs = frag + j * slot_u32;
    float* bs = bsum + j * bsum_slot;
    // one thread per 4 consecutive inputs (2 B-fragment pairs); 8 consecutive
    // threads cover one 32-input block, so Q4_1 block sums reduce by shuffles
    const int quads = geff * 64 * M;
    for (int idx = threadIdx.x; idx < quads; idx += blockDim.x) {
      const int r = idx / (geff * 64);
      const int rem = idx - r * geff * 64;
      const int cc = rem >> 6, q4 = rem & 63;
      const int k = kbase + cc * kChunkK + q4 * 4;
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (r < rows) {
        const float* xr = a.x + (size_t)r * a.ldx;
        if (k + 3 < a.k && ((((uintptr_t)(xr + k)) & 15) == 0)) {
          const float4 t = *reinterpret_cast<const float4*>(xr + k);
          v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
          for (int e = 0; e < 4; ++e)
            if (k + e < a.k) v[e] = xr[k + e];
        }
        if (NORM) {
          const float sc = inv_rms[r];
          for (int e = 0; e < 4; ++e)
            if (k + e < a.k) v[e] = __fmul_rn(__fmul_rn(v[e], sc), a.norm_w[k + e]);
        }
      }
      uint32_t* base = fs + cc * frag_chunk_u32<M>();
#pragma unroll
      for (int p2 = 0; p2 < 2; ++p2) {
        const int kk = q4 * 4 + p2 * 2;  // even input index inside the chunk
        const int st = kk >> 4, wv = kk & 15;
        const int reg = wv >= 8, cl = (wv & 7) >> 1;
        const __half h0 = __float2half_rn(v[2 * p2]), h1 = __float2half_rn(v[2 * p2 + 1]);
        const __half l0 = __float2half_rn(v[2 * p2] - __half2float(h0));
        const __half l1 = __float2half_rn(v[2 * p2 + 1] - __half2float(h1));
        const int lane_hi = 4 * (2 * r) + cl, lane_lo = lane_hi + 4;
        base[lane_hi * kFragLaneStride + st * 2 + reg] = h2_as_u32(__halves2half2(h0, h1));
        base[lane_lo * kFragLaneStride + st * 2 + reg] = h2_as_u32(__halves2half2(l0, l1));
      }
      if (QT == MLB_Q4_1) {
        float s4 = (v[0] + v[1]) + (v[2] + v[3]);
        s4 += __shfl_xor_sync(0xffffffffu, s4, 1);
        s4 += __shfl_xor_sync(0xffffffffu, s4, 2);
        s4 += __shfl_xor_sync(0xffffffffu, s4, 4);
        if ((q4 & 7) == 0) bs[(cc * 8 + (q4 >> 3)) * M + r] = s4;
      }
    }
  }
  __syncthreads();

  // 4. Stream this warp's super-blocks, accumulating per run.
  const int g = lane >> 2, cl = lane & 3;
  const bool bl = lane < 8 * M;  // lanes carrying B-fragment columns
  const int qbytes = QT == MLB_Q8_0 ? 4096 : 2048;
  float acc0 = 0.0f, acc1 = 0.0f;
  int b_chunk = -1, r = 0, last_r = -1;
  uint32_t B[16][2];
#pragma unroll
  for (int s = 0; s < 16; ++s) B[s][0] = B[s][1] = 0u;
  int slot = 0;
  uint32_t parity = 0;
  for (long long u = cb + warp; u < ce; u += kGemvWarps) {
    while (u >= run_u0[r + 1]) ++r;
    if (r != last_r) {
      if (last_r >= 0 && cl < M) {
        float* sl = slots + ((size_t)last_r * kGemvWarps + warp) * 16 * M;
        sl[g * M + cl] = acc0;
        sl[(g + 8) * M + cl] = acc1;
      }
      acc0 = acc1 = 0.0f;
      last_r = r;
    }
    const int grp = run_grp[r];
    const int cc = run_cc0[r] + (int)(u - run_u0[r]);
    const int chunk = grp * a.gc + cc;
    if (chunk != b_chunk) {
      b_chunk = chunk;
      if (bl) {
        const uint32_t* fsrc =
            frag + (grp - g0) * slot_u32 + cc * frag_chunk_u32<M>() + lane * kFragLaneStride;
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
    if (!mbar_wait_bounded(&mybars[slot], parity, a.status, 2)) return;
    const uint8_t* sb = myring + (size_t)slot * sbb;

    // everything this lane needs from the super-block, as 16-byte loads
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
    constexpr int kQLoads = QT == MLB_Q8_0 ? 8 : 4;  // uint4 per lane per super-block
    uint4 qv[kQLoads];
#pragma unroll
    for (int i = 0; i < kQLoads; ++i)
      qv[i] = *reinterpret_cast<const uint4*>(sb + (size_t)(i * 32 + lane) * 16);

#pragma unroll
    for (int b = 0; b < 8; ++b) {
      uint32_t A1[4], A2[4];
      if (QT == MLB_Q8_0) {
        const uint4 q = qv[b];
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
        const uint4 q = qv[b >> 1];
        const uint32_t w0 = (b & 1) ? q.z : q.x, w1 = (b & 1) ? q.w : q.y;  // rows g, g+8
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
        const float sx = bsum[(grp - g0) * bsum_slot + (cc * 8 + b) * M + rr];
        acc0 = fmaf(mn.x, sx, acc0);
        acc1 = fmaf(mn.y, sx, acc1);
      }
    }
    // All lanes have consumed the slot (their loads fed the MMAs above), so lane 0
    // can refill it; the mbarrier protocol orders the bulk copy after the reads.
    __syncwarp();
    const long long un = u + (long long)S * kGemvWarps;
    if (lane == 0 && un < ce) {
      mbar_arrive_expect_tx(&mybars[slot], sbb);
      bulk_g2s(myring + (size_t)slot * sbb, a.w + (size_t)un * sbb, sbb, &mybars[slot]);
    }
    if (++slot == S) {
      slot = 0;
      parity ^= 1u;
    }
  }
  if (last_r >= 0 && cl < M) {
    float* sl = slots + ((size_t)last_r * kGemvWarps + warp) * 16 * M;
    sl[g * M + cl] = acc0;
    sl[(g + 8) * M + cl] = acc1;
  }
  __syncthreads();

  // 5. Finish the runs: sum the warps' slots in warp order; a run that is a
  //    whole tile goes straight to the epilogue, a partial one joins the
  //    tile's other segments through the workspace (last arriver sums them in
  //    chunk order).
  float* myred = red + warp * (16 * M + kSegList);
  int* seglist = reinterpret_cast<int*>(myred + 16 * M);
  for (int rr = warp; rr < nruns; rr += kGemvWarps) {
    const int t = run_t[rr], grp = run_grp[rr];
    const int geff = min(a.gc, a.nchunks - grp * a.gc);
    const long long len = run_u0[rr + 1] - run_u0[rr];
    for (int i = lane; i < 16 * M; i += 32) {
      float s = 0.0f;
      for (int w = 0; w < kGemvWarps; ++w) s += slots[((size_t)rr * kGemvWarps + w) * 16 * M + i];
      myred[i] = s;
    }
    __syncwarp();
    bool finish = a.ngroups == 1 && run_cc0[rr] == 0 && len == geff;
    if (!finish) {
      float* slotw = a.ws + ((size_t)t * a.nchunks + grp * a.gc + run_cc0[rr]) * 16 * M;
      for (int i = lane; i < 16 * M; i += 32) slotw[i] = myred[i];
      __threadfence();
      __syncwarp();
      int nseg = 0;
      if (lane == 0)
        nseg = for_each_segment(t, a.ntiles, a.nchunks, a.gc, a.ngroups, a.nsb, G, [](int) {});
      int last = 0;
      if (lane == 0) last = (atomicAdd(&a.counters[t], 1) == nseg - 1);
      last = __shfl_sync(0xffffffffu, last, 0);
      finish = last != 0;
      if (finish) {
        __threadfence();
        float s[(16 * M + 31) / 32];
#pragma unroll
        for (int q = 0; q < (16 * M + 31) / 32; ++q) s[q] = 0.0f;
        // gather the segment starts kSegList at a time, then sum with
        // independent loads, in chunk order
        int done = 0;
        while (true) {
          int cnt = 0;
          if (lane == 0) {
            int idx = 0;
            for_each_segment(t, a.ntiles, a.nchunks, a.gc, a.ngroups, a.nsb, G, [&](int c) {
              if (idx >= done && idx < done + kSegList) seglist[idx - done] = c;
              ++idx;
            });
            cnt = min(kSegList, idx - done);
          }
          cnt = __shfl_sync(0xffffffffu, cnt, 0);
          __syncwarp();
          if (cnt <= 0) break;
#pragma unroll
          for (int q = 0; q < (16 * M + 31) / 32; ++q) {
            const int i = lane + 32 * q;
            if (i < 16 * M)
              for (int j = 0; j < cnt; ++j)
                s[q] += __ldcg(a.ws + ((size_t)t * a.nchunks + seglist[j]) * 16 * M + i);
          }
          done += cnt;
          __syncwarp();
          if (cnt < kSegList) break;
        }
#pragma unroll
        for (int q = 0; q < (16 * M + 31) / 32; ++q) {
          const int i = lane + 32 * q;
          if (i < 16 * M) myred[i] = s[q];
        }
        if (lane == 0) a.counters[t] = 0;
        __syncwarp();
      }
    }
    if (finish) {
      for (int i = lane; i < 16 * M; i += 32) {
        int row = i / M, rb = i - row * M;
        if (rb < rows) epilogue_row<M>(a.epi, t, row, rb, myred);
      }
      if (a.epi.argmax_key) {
        unsigned long long key = 0ull;
        if (lane < 16 && t * 16 + lane < a.epi.n_out)
          key = argmax_key_of(myred[lane * M], a.epi.argmax_base + t * 16 + lane);
        key = warp_max_u64(key);
        if (lane == 0 && key) atomicMax(a.epi.argmax_key, key);
      }
    }
    __syncwarp();
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

// Largest number of (group, tile) runs, and of chunk groups, any CTA range
// touches when the super-blocks are split over G CTAs.
static void cta_span(const QMatrix& m, long long G, int* max_runs, int* max_groups) {
  *max_runs = 0;
  *max_groups = 0;
  for (long long c = 0; c < G; ++c) {
    long long u = cta_start(c, m.nsb, G);
    const long long ce = cta_start(c + 1, m.nsb, G);
    int runs = 0, g0 = -1, g1 = -1;
    while (u < ce) {
      const SbPos sp = sb_decode(u, m.ntiles, m.nchunks, m.gc);
      if (g0 < 0) g0 = sp.grp;
      g1 = sp.grp;
      u += std::min((long long)(sp.geff - sp.cc), ce - u);
      ++runs;
    }
    *max_runs = std::max(*max_runs, runs);
    *max_groups = std::max(*max_groups, g0 < 0 ? 0 : g1 - g0 + 1);
  }
}

// Grid for a matrix: one CTA per SM unless a CTA range would touch more runs
// or chunk groups than its shared memory holds; then whole extra waves of
// (smaller) CTAs, since only one CTA fits on an SM.
template <int M>
static long long choose_grid(const QMatrix& m, int sms) {
  const int idx = M == 1 ? 0 : (M == 2 ? 1 : 2);
  if (m.grid_cache[idx] > 0) return m.grid_cache[idx];
  long long G = std::min<long long>(std::max<long long>(sms, m.ngroups > 1 ? m.ngroups + 1 : 1),
                                    m.nsb);
  while (true) {
    int runs = 0, groups = 0;
    cta_span(m, G, &runs, &groups);
    if ((runs <= max_cta_runs<M>() && groups <= 2) || G >= m.nsb) break;
    G = std::min<long long>(m.nsb, (G / sms + 1) * sms);
  }
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
      kMaxStages, fixed < kSmemMax ? (kSmemMax - fixed) / ((size_t)kGemvWarps * sbb) : 0);
  if (stages < 2) invalid("gemv: staged activations leave no room for the weight ring");
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

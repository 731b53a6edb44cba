// gemv_dev.cuh — device building blocks of the super-block GEMV, shared by the
// standalone GEMV kernel (gemv.cu) and the persistent decode-step kernel
// (step.cu), so both compute every output with the same instructions in the
// same order.
//
// Work split. A matrix of nsb super-blocks (SB) is cut into G contiguous CTA
// ranges [cta_start(c), cta_start(c + 1)) of whole group-tiles (the SBs of one
// tile within one chunk group). Inside a range, warp w takes SBs cb + w,
// cb + w + 16, ... Each group-tile of the range is a "run"; each warp keeps
// one fp32 partial per run and row, and the CTA sums the 16 warps' partials of
// a run in warp order. When K fits one chunk group (every decode shape up to
// K = 16384) a run is a whole tile and goes straight to the epilogue, with no
// traffic between CTAs; otherwise the last of a tile's per-group segments to
// arrive sums them in chunk order. Results are therefore deterministic and
// independent of timing.
#pragma once

#include <cuda_bf16.h>

#include "gemv.cuh"

namespace mlb {

constexpr int kFragLaneStride = 36;  // u32 per lane per chunk (32 + 4 pad: no bank conflicts)
constexpr int kSegList = 32;         // segment starts gathered per pass of a fix-up

template <int M>
__host__ __device__ constexpr int frag_chunk_u32() {
  return 8 * M * kFragLaneStride;
}
// A CTA range is processed in windows of at most kWinRuns runs (group-tiles)
// and win_sbs<M>() super-blocks, ending at run boundaries; each super-block of
// a window leaves its 16 x M partial dot products in shared memory (16 KB).
constexpr int kWinRuns = 64;
template <int M>
__host__ __device__ constexpr int win_sbs() {
  return 256 / M;
}

// Side data per staged chunk: [8 blocks][M] bias corrections (see
// sb_accumulate), then for Q4_1 [8 blocks][M] block sums of x.
template <int QT, int M>
__host__ __device__ constexpr int side_per_chunk() {
  return 8 * M * (QT == MLB_Q4_1 ? 2 : 1);
}

struct SbPos {
  int grp, t, cc, geff;
};

// Device geometry is 32-bit throughout: super-block and group-tile counts of
// any decode matrix stay far below 2^31 (and products such as ngt * c below
// 2^31 for grids of <= 256 CTAs), and 64-bit division is a long emulated
// sequence on the GPU.
__host__ __device__ inline SbPos sb_decode(int u, int ntiles, int nchunks, int gc) {
  SbPos s;
  const int per = ntiles * gc;
  s.grp = u / per;
  const int rem = u - s.grp * per;
  s.geff = min(gc, nchunks - s.grp * gc);
  s.t = rem / s.geff;
  s.cc = rem - s.t * s.geff;
  return s;
}

// Group-tiles: the (chunk group, tile) pairs in super-block order; group-tile
// gt = grp * ntiles + t is the geff consecutive super-blocks of tile t in
// group grp. CTA c of G owns group-tiles [ngt c / G, ngt (c + 1) / G), i.e.
// whole tiles of each chunk group, so a tile is computed inside one CTA except
// for its split over chunk groups (K beyond one group only).
__host__ __device__ inline int gt_sb_start(int gt, int ntiles, int nchunks, int gc) {
  const int ngt = ((nchunks + gc - 1) / gc) * ntiles;
  if (gt >= ngt) return ntiles * nchunks;
  const int grp = gt / ntiles, t = gt - grp * ntiles;
  const int geff = min(gc, nchunks - grp * gc);
  return grp * ntiles * gc + t * geff;
}

// First super-block of CTA c's range (c = G gives the end of the matrix).
__host__ __device__ inline int cta_start(int c, int G, int ntiles, int nchunks, int gc,
                                         int ngroups) {
  const int ngt = ngroups * ntiles;
  return gt_sb_start(ngt * c / G, ntiles, nchunks, gc);
}

// Calls f(start_chunk) for every segment tile t is split into (one per chunk
// group, in chunk order); returns the segment count.
template <class F>
__device__ __forceinline__ int for_each_segment(int ngroups, int gc, F f) {
  for (int gr = 0; gr < ngroups; ++gr) f(gr * gc);
  return ngroups;
}

// Run table of one CTA range, in shared memory: run i is the SBs
// [u0[i], u0[i + 1]) of tile t[i] in chunk group grp[i], starting at chunk cc0[i]
// of the group.
struct RunTable {
  int* u0;        // [R + 1]
  int* t;         // [R]
  int* grp;       // [R]
  int* cc0;       // [R]
};

// One thread: fills the run table of the window that starts at wb in a CTA
// range ending at ce: whole group-tiles, at most R of them and at most maxsb
// super-blocks (a group-tile is never longer than maxsb). Returns the run
// count; the window ends at rt.u0[count].
__device__ __forceinline__ int build_window(int wb, int ce, int ntiles, int nchunks, int gc,
                                            int R, int maxsb, const RunTable& rt) {
  int u = wb;
  int r = 0;
  SbPos sp = sb_decode(u, ntiles, nchunks, gc);  // one decode; then walk run by run
  while (u < ce && r < R) {
    const int len = min(sp.geff - sp.cc, ce - u);
    if (r > 0 && u + len - wb > maxsb) break;
    rt.u0[r] = u;
    rt.t[r] = sp.t;
    rt.grp[r] = sp.grp;
    rt.cc0[r] = sp.cc;
    u += len;
    ++r;
    sp.cc = 0;  // the next run starts a group-tile
    if (++sp.t == ntiles) {
      sp.t = 0;
      ++sp.grp;
      sp.geff = min(gc, nchunks - sp.grp * gc);
    }
  }
  rt.u0[r] = u;
  return r;
}

// Block-wide form of build_window. With one chunk group every run is a whole
// tile of nchunks super-blocks, so run r of the window starts at wb + r
// nchunks and thread r fills entry r (no serial walk); with several groups
// thread 0 walks. *nruns is written by thread 0. Visible after the caller's
// __syncthreads.
__device__ __forceinline__ void build_window_par(int wb, int ce, int ntiles, int nchunks, int gc,
                                                 int ngroups, int R, int maxsb,
                                                 const RunTable& rt, int* nruns) {
  if (ngroups > 1) {
    if (threadIdx.x == 0) *nruns = build_window(wb, ce, ntiles, nchunks, gc, R, maxsb, rt);
    return;
  }
  const int n = max(1, min(min((ce - wb) / nchunks, R), maxsb / nchunks));
  const int t0 = wb / nchunks;  // wb starts a tile
  for (int r = threadIdx.x; r <= n; r += blockDim.x) {
    rt.u0[r] = wb + r * nchunks;
    if (r < n) {
      rt.t[r] = t0 + r;
      rt.grp[r] = 0;
      rt.cc0[r] = 0;
    }
  }
  if (threadIdx.x == 0) *nruns = n;
}

// A warp's position in the super-block order, advanced 16 super-blocks at a
// time without divisions: chunk cc of tile t in chunk group grp (geff chunks),
// and the offsets of that chunk's staged B fragments and side data.
struct SbCursor {
  int cc, t, grp, geff;
  int fofs, sofs;
};

template <int QT, int M>
__device__ __forceinline__ void cursor_set(SbCursor& c, int u, int ntiles, int nchunks,
                                           int gc, int g0) {
  const SbPos sp = sb_decode(u, ntiles, nchunks, gc);
  c.cc = sp.cc;
  c.t = sp.t;
  c.grp = sp.grp;
  c.geff = sp.geff;
  c.fofs = ((c.grp - g0) * gc + c.cc) * frag_chunk_u32<M>();
  c.sofs = ((c.grp - g0) * gc + c.cc) * side_per_chunk<QT, M>();
}

// Stepping past the end of the matrix leaves the cursor in the last chunk
// group's range of values (it is not used again): every loop here advances.
template <int QT, int M>
__device__ __forceinline__ void cursor_step16(SbCursor& c, int ntiles, int nchunks, int gc,
                                              int g0) {
  c.cc += kGemvWarps;
  while (c.cc >= c.geff) {
    c.cc -= c.geff;
    if (++c.t == ntiles) {
      c.t = 0;
      if ((c.grp + 1) * gc >= nchunks) {  // no chunk group left: park the cursor
        c.cc = 0;
        break;
      }
      ++c.grp;
      c.geff = min(gc, nchunks - c.grp * gc);
    }
  }
  const int ch = (c.grp - g0) * gc + c.cc;
  c.fofs = ch * frag_chunk_u32<M>();
  c.sofs = ch * side_per_chunk<QT, M>();
}

// --------------------------------------------------------------- epilogues

template <int M>
// Returns the value stored for a residual row (0 for other kinds).
__device__ float epilogue_row(const EpiParams& p, int tile, int row, int r, const float* vals) {
  float v = vals[row * M + r];
  int grow = tile * 16 + row;
  switch (p.kind) {
    case kEpiStore:
      if (grow < p.n_out) {
        if (p.tp) {
          const long long o = p.tp->logits_off + (long long)(p.argmax_base + grow) * 4;
          for (int rr = 0; rr < p.tp->n; ++rr) *reinterpret_cast<float*>(p.tp->peers[rr] + o) = v;
        } else {
          p.y[(size_t)r * p.ldy + grow] = v;
        }
      }
      break;
    case kEpiTpPartial:
      if (grow < p.n_out) {
        const TpXchg* x = p.tp;
        const long long o =
            x->parts_off + ((long long)(p.tp_slot * x->n + x->me) * x->dim + grow) * 8;
        const unsigned long long word =
            ((unsigned long long)p.tp_tag << 32) | (unsigned long long)__float_as_uint(v);
        for (int rr = 0; rr < x->n; ++rr)  // one whole 8-byte word per rank
          asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(x->peers[rr] + o), "l"(word)
                       : "memory");
      }
      break;
    case kEpiResidual:
      if (grow < p.n_out) {
        const float rv = p.resid_s ? p.resid_s[grow - p.resid_t0 * 16]
                                   : __ldcg(p.resid + (size_t)r * p.ldr + grow);
        const float y = __fadd_rn(rv, v);
        p.y[(size_t)r * p.ldy + grow] = y;
        return y;
      }
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
      int pos = p.pos_set ? p.pos_now : *p.pos;
      if (sec == 2) {
        if (p.kv_bf16)
          reinterpret_cast<__nv_bfloat16*>(p.values)[(size_t)pos * p.kv_rows + L] =
              __float2bfloat16_rn(v);
        else
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
      float2 cs = p.rope_s ? p.rope_s[j] : p.rope[(size_t)pos * (D / 2) + j];
      float out;
      if (first)  // a*c - b*s with a = this, b = partner (src/ops.cc:155, 174)
        out = __fsub_rn(__fmul_rn(v, cs.x), __fmul_rn(w, cs.y));
      else        // a*s + b*c with a = partner, b = this (src/ops.cc:156, 175)
        out = __fadd_rn(__fmul_rn(w, cs.y), __fmul_rn(v, cs.x));
      if (sec == 0)
        p.q_out[(size_t)r * p.q_rows + L] = out;
      else if (p.kv_bf16)
        reinterpret_cast<__nv_bfloat16*>(p.keys)[(size_t)pos * p.kv_rows + L] =
            __float2bfloat16_rn(out);
      else
        p.keys[(size_t)pos * p.kv_rows + L] = out;
      break;
    }
  }
  return 0.0f;
}

// ------------------------------------------------------ activation staging

// Block-wide: inv_rms[r] = 1 / sqrt(sum(x_r^2) / K + eps) for r < rows, the
// RMSNorm statistic of src/ops.cc:55-61 (per-thread strided sums, warp trees,
// then the 16 warp sums in warp order). part: [kGemvWarps] scratch.
// Starts and ends with the block synchronised.
__device__ __forceinline__ void norm_inv_rms(const float* x, int ldx, int rows, int k, float eps,
                                             float* part, float* inv_rms) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = 0; r < rows; ++r) {
    float ss = 0.0f;
    const float* xr = x + (size_t)r * ldx;
    if ((k & 3) == 0 && (((uintptr_t)xr) & 15) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      for (int i = threadIdx.x; i < (k >> 2); i += blockDim.x) {
        const float4 v = __ldcg(x4 + i);
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
      }
    } else {
      for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const float v = __ldcg(xr + i);
        ss = fmaf(v, v, ss);
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) part[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.0f;
      for (int w = 0; w < kGemvWarps; ++w) t += part[w];  // fixed order
      t = __fdiv_rn(t, (float)k);
      inv_rms[r] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(t, eps)));
    }
    __syncthreads();
  }
}

// Writes four consecutive inputs e (chunk inputs 4 q4 .. 4 q4 + 3 of batch row
// r) into the chunk's B fragments as fp16 hi + lo, and returns their part of
// the block's bias correction. The Q4 formats stage the inputs of block
// positions 16..31 divided by 16 (a power of two: exact), because the high
// nibbles enter the MMA as 1024 + 16 q; the correction is the bias times the
// staged (represented) values: Q4_0 1032 (positions 0..15) and 1152 (16..31),
// Q4_1 1024, Q8_0 1152.
template <int QT, int M>
__device__ __forceinline__ float stage_quad(uint32_t* cbase, int r, int q4, const float (&e)[4]) {
  const bool upper = (q4 & 7) >= 4;  // block positions 16..31
  const float f = (QT != MLB_Q8_0 && upper) ? 0.0625f : 1.0f;
  float rep = 0.0f;
#pragma unroll
  for (int p2 = 0; p2 < 2; ++p2) {
    const int kk = q4 * 4 + p2 * 2;  // even input index inside the chunk
    const int st = kk >> 4, wv = kk & 15;
    const int reg = wv >= 8, cl = (wv & 7) >> 1;
    const float v0 = e[2 * p2] * f, v1 = e[2 * p2 + 1] * f;
    const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
    const __half l0 = __float2half_rn(v0 - __half2float(h0));
    const __half l1 = __float2half_rn(v1 - __half2float(h1));
    const int lane_hi = 4 * (2 * r) + cl, lane_lo = lane_hi + 4;
    cbase[lane_hi * kFragLaneStride + st * 2 + reg] = h2_as_u32(__halves2half2(h0, h1));
    cbase[lane_lo * kFragLaneStride + st * 2 + reg] = h2_as_u32(__halves2half2(l0, l1));
    rep += (__half2float(h0) + __half2float(l0)) + (__half2float(h1) + __half2float(l1));
  }
  const float bias = QT == MLB_Q4_0 ? (upper ? 1152.0f : 1032.0f)
                                    : (QT == MLB_Q4_1 ? 1024.0f : 1152.0f);
  return bias * rep;
}

// Sums a per-quad value over the 8 lanes of one 32-input block (lanes 8i ..
// 8i + 7, shuffle tree: fixed order). Every lane of the warp must call it.
__device__ __forceinline__ float block_sum8(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  return v;
}

// Block-wide: x (normalised with inv_rms and norm_w when norm_w is non-null)
// of chunk groups g0..g1 into the mma B-fragment layout (fp16 hi in column 2r,
// fp16 lo in column 2r + 1 of batch row r) with the chunk side data. Rows >=
// rows and inputs >= k stage as zero. The caller synchronises afterwards.
template <int QT, int M>
__device__ __forceinline__ void stage_x(const float* x, int ldx, int rows, int k,
                                        const float* norm_w, const float* inv_rms, int gc,
                                        int nchunks, int g0, int g1, uint32_t* frag,
                                        float* side) {
  constexpr int SPC = side_per_chunk<QT, M>();
  const int slot_u32 = gc * frag_chunk_u32<M>();
  for (int j = 0; j <= g1 - g0; ++j) {
    const int grp = g0 + j;
    const int geff = min(gc, nchunks - grp * gc);
    const int kbase = grp * gc * kChunkK;
    uint32_t* fs = frag + j * slot_u32;
    float* sd = side + (size_t)j * gc * SPC;
    // one thread per 4 consecutive inputs (2 B-fragment pairs); 8 consecutive
    // threads cover one 32-input block, so block sums reduce by shuffles
    const int quads = geff * 64 * M;
    for (int idx = threadIdx.x; idx < quads; idx += blockDim.x) {
      const int r = idx / (geff * 64);
      const int rem = idx - r * geff * 64;
      const int cc = rem >> 6, q4 = rem & 63;
      const int kk0 = kbase + cc * kChunkK + q4 * 4;
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (r < rows) {
        const float* xr = x + (size_t)r * ldx;
        if (kk0 + 3 < k && ((((uintptr_t)(xr + kk0)) & 15) == 0)) {
          const float4 t = __ldcg(reinterpret_cast<const float4*>(xr + kk0));
          v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
          for (int e = 0; e < 4; ++e)
            if (kk0 + e < k) v[e] = __ldcg(xr + kk0 + e);
        }
        if (norm_w) {
          const float sc = inv_rms[r];
          for (int e = 0; e < 4; ++e)
            if (kk0 + e < k) v[e] = __fmul_rn(__fmul_rn(v[e], sc), norm_w[kk0 + e]);
        }
      }
      const float corr = block_sum8(stage_quad<QT, M>(fs + cc * frag_chunk_u32<M>(), r, q4, v));
      float* sc = sd + cc * SPC;
      if ((q4 & 7) == 0) sc[(q4 >> 3) * M + r] = corr;
      if (QT == MLB_Q4_1) {
        const float s4 = block_sum8((v[0] + v[1]) + (v[2] + v[3]));
        if ((q4 & 7) == 0) sc[8 * M + (q4 >> 3) * M + r] = s4;
      }
    }
  }
}

// Four consecutive inputs from k0 of a row of length k (zeros past the end).
__device__ __forceinline__ float4 load_quad(const float* row, int k0, int k, bool cached) {
  if (k0 + 3 < k && ((((uintptr_t)(row + k0)) & 15) == 0))
    return cached ? __ldg(reinterpret_cast<const float4*>(row + k0))
                  : __ldcg(reinterpret_cast<const float4*>(row + k0));
  float e[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int i = 0; i < 4; ++i)
    if (k0 + i < k) e[i] = cached ? __ldg(row + k0 + i) : __ldcg(row + k0 + i);
  return make_float4(e[0], e[1], e[2], e[3]);
}

constexpr int kStageBatch = 4;  // float4 of x each thread loads per round trip

// Block-wide, one batch row: stage_x with the RMSNorm statistic formed in the
// same pass. Each thread loads its float4s of x (and of the norm weight) for
// kStageBatch rounds at once, so staging costs one round trip to L2 per
// kStageBatch * blockDim float4. With a norm and all of K within one batch
// (K <= 8192 at 512 threads) the statistic comes from those registers: each
// thread's float4 i = tid, tid + blockDim, ... summed in order, warp trees,
// then the warp sums in warp order, the same order as norm_inv_rms; longer
// rows take norm_inv_rms's extra pass. A norm needs the CTA to stage all of K
// (g0 .. g1 cover every chunk group). The caller synchronises afterwards.
template <int QT>
__device__ __forceinline__ void stage_x_m1(const float* x, int k, const float* norm_w, float eps,
                                           int gc, int nchunks, int g0, int g1, uint32_t* frag,
                                           float* side, float* part, float* inv_rms) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nthr = blockDim.x;
  const int c0 = g0 * gc, c1 = min(nchunks, (g1 + 1) * gc);
  const int nq = (c1 - c0) * 64;
  const int kbase = c0 * kChunkK;
  const int slot_u32 = gc * frag_chunk_u32<1>();
  const bool fused = norm_w != nullptr && c0 == 0 && c1 == nchunks && nq <= kStageBatch * nthr;
  if (norm_w && !fused) norm_inv_rms(x, k, 1, k, eps, part, inv_rms);
  for (int base = 0; base < nq; base += kStageBatch * nthr) {
    float4 v[kStageBatch], w[kStageBatch];
#pragma unroll
    for (int j = 0; j < kStageBatch; ++j) {
      const int idx = base + j * nthr + threadIdx.x;
      v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      w[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (idx < nq) {
        v[j] = load_quad(x, kbase + idx * 4, k, false);
        if (norm_w) w[j] = load_quad(norm_w, kbase + idx * 4, k, true);
      }
    }
    if (fused) {
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        ss = fmaf(v[j].x, v[j].x, ss);
        ss = fmaf(v[j].y, v[j].y, ss);
        ss = fmaf(v[j].z, v[j].z, ss);
        ss = fmaf(v[j].w, v[j].w, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) part[warp] = ss;
      __syncthreads();
      if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < (nthr >> 5); ++i) t += part[i];  // fixed order
        t = __fdiv_rn(t, (float)k);
        inv_rms[0] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(t, eps)));
      }
      __syncthreads();
    }
    const float sc = norm_w ? inv_rms[0] : 1.0f;
#pragma unroll
    for (int j = 0; j < kStageBatch; ++j) {
      const int idx = base + j * nthr + threadIdx.x;
      const bool valid = idx < nq;  // uniform over each 8-lane block group
      float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      if (norm_w) {
        const float wv[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) e[i] = __fmul_rn(__fmul_rn(e[i], sc), wv[i]);
      }
      const int chunk = c0 + (idx >> 6), q4 = idx & 63;
      const int grp = chunk / gc, cc = chunk - grp * gc;
      float corr = 0.0f;
      if (valid)
        corr = stage_quad<QT, 1>(frag + (grp - g0) * slot_u32 + cc * frag_chunk_u32<1>(), 0, q4,
                                 e);
      corr = block_sum8(corr);
      float* sd = side + ((size_t)(grp - g0) * gc + cc) * side_per_chunk<QT, 1>();
      if (valid && (q4 & 7) == 0) sd[q4 >> 3] = corr;
      if (QT == MLB_Q4_1) {
        const float s4 = block_sum8((e[0] + e[1]) + (e[2] + e[3]));
        if (valid && (q4 & 7) == 0) sd[8 + (q4 >> 3)] = s4;
      }
    }
  }
}

// The B fragments of one staged chunk for this lane (16 k-steps x 2 regs).
__device__ __forceinline__ void load_b(const uint32_t* fsrc_lane, uint32_t (&B)[16][2]) {
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    uint4 v = *reinterpret_cast<const uint4*>(fsrc_lane + s * 4);
    B[2 * s][0] = v.x;
    B[2 * s][1] = v.y;
    B[2 * s + 1][0] = v.z;
    B[2 * s + 1][1] = v.w;
  }
}

// ------------------------------------------------ one super-block, one warp

// acc0 / acc1 (rows g and g + 8 of the tile, batch row lane & 3 when < M)
// += the super-block in shared memory times the staged chunk in B.
// side_chunk: the chunk's side data (side_per_chunk).
//
// The codes are decoded through the magic exponent: a 4-bit code ORed into
// the mantissa of 1024.0h is exactly 1024 + q (low nibble) or 1024 + 16 q
// (high nibble, whose activations were staged divided by 16); an int8 code
// through prmt is 1024 + 128 + q. One half2 subtraction per register then
// leaves the exact small integers q - 8 (Q4_0), q (Q4_1) or the int8 value
// (Q8_0), so each block's fp32 MMA chain is the block dot itself (its
// rounding relative to that dot, as in the reference's sequential fp32 sum).
template <int QT, int M>
__device__ __forceinline__ void sb_accumulate(const uint8_t* sb, int lane,
                                              const uint32_t (&B)[16][2],
                                              const float* side_chunk, float& acc0,
                                              float& acc1) {
  const int g = lane >> 2, cl = lane & 3;
  const int rr = cl < M ? cl : 0;
  constexpr int qbytes = QT == MLB_Q8_0 ? 4096 : 2048;
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
      const uint32_t wx[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                              q.w ^ 0x80808080u};
      // wx[0]: row g (k 2c,2c+1,2c+8,2c+9), wx[1]: row g (+16), wx[2..3]: row g+8
      A1[0] = __byte_perm(wx[0], 0x64646464u, 0x4140);
      A1[2] = __byte_perm(wx[0], 0x64646464u, 0x4342);
      A1[1] = __byte_perm(wx[2], 0x64646464u, 0x4140);
      A1[3] = __byte_perm(wx[2], 0x64646464u, 0x4342);
      A2[0] = __byte_perm(wx[1], 0x64646464u, 0x4140);
      A2[2] = __byte_perm(wx[1], 0x64646464u, 0x4342);
      A2[1] = __byte_perm(wx[3], 0x64646464u, 0x4140);
      A2[3] = __byte_perm(wx[3], 0x64646464u, 0x4342);
    } else {
      const uint4 q = qv[b >> 1];
      const uint32_t w0 = (b & 1) ? q.z : q.x, w1 = (b & 1) ? q.w : q.y;  // rows g, g+8
      const uint32_t w0s = w0 >> 8, w1s = w1 >> 8;
      const uint32_t M1 = 0x000F000Fu, M2 = 0x00F000F0u, E = 0x64006400u;
      // low nibbles: 1024 + q ; high nibbles: 1024 + 16 q
      A1[0] = lop3_and_or(w0, M1, E);
      A1[1] = lop3_and_or(w1, M1, E);
      A1[2] = lop3_and_or(w0s, M1, E);
      A1[3] = lop3_and_or(w1s, M1, E);
      A2[0] = lop3_and_or(w0, M2, E);
      A2[1] = lop3_and_or(w1, M2, E);
      A2[2] = lop3_and_or(w0s, M2, E);
      A2[3] = lop3_and_or(w1s, M2, E);
    }
    // remove the magic bias in fp16 (exact: small integers), so the MMA sums
    // the codes' own products and its fp32 rounding is relative to the block
    // dot itself rather than to ~1000 times the block sum of x
    {
      const __half2 b1 = __float2half2_rn(QT == MLB_Q4_0 ? 1032.0f
                                                        : (QT == MLB_Q4_1 ? 1024.0f : 1152.0f));
      const __half2 b2 = __float2half2_rn(QT == MLB_Q4_0 ? 1152.0f
                                                        : (QT == MLB_Q4_1 ? 1024.0f : 1152.0f));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        A1[i] = h2_as_u32(__hsub2(u32_as_h2(A1[i]), b1));
        A2[i] = h2_as_u32(__hsub2(u32_as_h2(A2[i]), b2));
      }
    }
    float d[4];
    mma_16816_z(d, A1, B[2 * b][0], B[2 * b][1]);
    mma_16816(d, A2, B[2 * b + 1][0], B[2 * b + 1][1]);
    const float2 sc = __half22float2(u32_as_h2(scw[b]));
    acc0 = fmaf(sc.x, d[0] + d[1], acc0);
    acc1 = fmaf(sc.y, d[2] + d[3], acc1);
    if (QT == MLB_Q4_1) {
      const float2 mn = __half22float2(u32_as_h2(mnw[b]));
      const float sx = side_chunk[8 * M + b * M + rr];
      acc0 = fmaf(mn.x, sx, acc0);
      acc1 = fmaf(mn.y, sx, acc1);
    }
  }
}

// One super-block's partial dot products: rows g and g + 8 of its tile, batch
// row cl (lanes with cl < M), at window-relative super-block index p.
template <int M>
__device__ __forceinline__ void store_sb_partial(float* parts, int p, int lane, float acc0,
                                                 float acc1) {
  const int g = lane >> 2, cl = lane & 3;
  if (cl < M) {
    float* pp = parts + (size_t)p * 16 * M;
    pp[g * M + cl] = acc0;
    pp[(g + 8) * M + cl] = acc1;
  }
}

// ---------------------------------------------------------- finishing runs

// Geometry of the matrix a CTA is finishing.
struct FinishGeom {
  int ntiles, nchunks, gc, ngroups;
  int rows;
};

// Block-wide, after a window's super-block partials are in parts and the block
// is synchronised: each run (one tile's super-blocks in one chunk group) sums
// its partials in chunk order. With one chunk group that is the tile's result
// and goes to the epilogue; otherwise it is written to the workspace and the
// last of the tile's group segments to arrive sums them in chunk order and
// runs the epilogue. red: [kGemvWarps][16 M + kSegList] scratch.
template <int M>
__device__ __forceinline__ void finish_runs(const float* parts, float* red, const RunTable& rt,
                                            int nruns, int wb, const FinishGeom& fg,
                                            float* ws, int* counters, const EpiParams& epi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* myred = red + warp * (16 * M + kSegList);
  int* seglist = reinterpret_cast<int*>(myred + 16 * M);
  for (int rr = warp; rr < nruns; rr += kGemvWarps) {
    const int t = rt.t[rr], grp = rt.grp[rr];
    const int p0 = rt.u0[rr] - wb, len = rt.u0[rr + 1] - rt.u0[rr];
    if (M == 1) {
      // one row per lane pair: lane r sums the first half of the row's
      // partials, lane r + 16 the second; the halves add in that order
      const int i = lane & 15, half = len >> 1;
      const int j0 = lane < 16 ? 0 : half, j1 = lane < 16 ? half : len;
      float s = 0.0f;
      for (int j = j0; j < j1; ++j) s += parts[(size_t)(p0 + j) * 16 + i];
      const float hi = __shfl_down_sync(0xffffffffu, s, 16);
      if (lane < 16) myred[i] = s + hi;
    } else {
      for (int i = lane; i < 16 * M; i += 32) {
        float s = 0.0f;
        for (int j = 0; j < len; ++j) s += parts[(size_t)(p0 + j) * 16 * M + i];
        myred[i] = s;
      }
    }
    __syncwarp();
    bool finish = fg.ngroups == 1;
    if (!finish) {
      float* slotw = ws + ((size_t)t * fg.nchunks + grp * fg.gc + rt.cc0[rr]) * 16 * M;
      for (int i = lane; i < 16 * M; i += 32) slotw[i] = myred[i];
      __threadfence();
      __syncwarp();
      int nseg = 0;
      if (lane == 0) nseg = for_each_segment(fg.ngroups, fg.gc, [](int) {});
      int last = 0;
      if (lane == 0) last = (atomicAdd(&counters[t], 1) == nseg - 1);
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
            for_each_segment(fg.ngroups, fg.gc, [&](int c) {
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
                s[q] += __ldcg(ws + ((size_t)t * fg.nchunks + seglist[j]) * 16 * M + i);
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
        if (lane == 0) counters[t] = 0;
        __syncwarp();
      }
    }
    if (finish) {
      float stored = 0.0f;  // M == 1: row `lane` (< 16) of the tile
      for (int i = lane; i < 16 * M; i += 32) {
        int row = i / M, rb = i - row * M;
        if (rb < fg.rows) stored = epilogue_row<M>(epi, t, row, rb, myred);
      }
      if (M == 1 && epi.ss_out && epi.kind == kEpiResidual) {
        // lane r < 16 stored row r above; its square, summed over the 16 rows
        // by a fixed tree (lanes 16.. add zeros and are not read)
        float sq = 0.0f;
        if (lane < 16 && t * 16 + lane < epi.n_out) sq = stored * stored;
        sq += __shfl_xor_sync(0xffffffffu, sq, 8);
        sq += __shfl_xor_sync(0xffffffffu, sq, 4);
        sq += __shfl_xor_sync(0xffffffffu, sq, 2);
        sq += __shfl_xor_sync(0xffffffffu, sq, 1);
        if (lane == 0) epi.ss_out[t] = sq;
      }
      if (epi.argmax_key) {
        unsigned long long key = 0ull;
        if (lane < 16 && t * 16 + lane < epi.n_out)
          key = argmax_key_of(myred[lane * M], epi.argmax_base + t * 16 + lane);
        key = warp_max_u64(key);
        if (lane == 0 && key) atomicMax(epi.argmax_key, key);
      }
    }
    __syncwarp();
  }
}

// Consumes one window [wb, we) of a warp's weight stream: the super-blocks
// u = cb + warp (mod 16) of the CTA range starting at cb, from the ring slot sequence
// (slot, parity), accumulating each against the staged x and leaving its
// partial in parts. After each slot is read, refill(slot) lets lane 0 reuse it
// for the next super-block of the warp's stream (and counts it in inflight,
// which lane 0 keeps). Returns false (warp-uniform) when a wait gave up.
template <int QT, int M, class Refill>
__device__ __forceinline__ bool consume_window(int cb, int wb, int we, int ntiles,
                                               int nchunks, int gc, int g0,
                                               const uint32_t* frag, const float* side,
                                               float* parts, uint8_t* ring, uint64_t* bars,
                                               int stride, int stages, int& slot,
                                               uint32_t& parity, int& inflight,
                                               DeviceStatus* status, int where, Refill& refill) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lag = (wb - cb) % kGemvWarps;
  const int u0 = wb + ((warp - lag + kGemvWarps) % kGemvWarps);
  if (u0 >= we) return true;
  const int n = (we - u0 + kGemvWarps - 1) / kGemvWarps;
  const int fl = lane < 8 * M ? lane : (lane & (8 * M - 1));  // lanes past the B columns: any valid data
  SbCursor c;
  cursor_set<QT, M>(c, u0, ntiles, nchunks, gc, g0);
  uint32_t B[16][2];
  int b_ofs = -1;
  float* pp = parts + (size_t)(u0 - wb) * 16 * M;
  for (int i = 0; i < n; ++i) {
    if (c.fofs != b_ofs) {
      b_ofs = c.fofs;
      load_b(frag + c.fofs + fl * kFragLaneStride, B);
    }
    uint64_t* bar = bars + slot;
    if (!mbar_try_wait(bar, parity) && !mbar_wait_bounded(bar, parity, status, where))
      return false;
    float acc0 = 0.0f, acc1 = 0.0f;
    sb_accumulate<QT, M>(ring + (size_t)slot * stride, lane, B, side + c.sofs, acc0, acc1);
    store_sb_partial<M>(pp, 0, lane, acc0, acc1);
    pp += 16 * kGemvWarps * M;
    // every lane has read the slot; lane 0 reuses it for the stream's next
    // super-block (the mbarrier orders the copy after the reads)
    __syncwarp();
    if (lane == 0) {
      --inflight;
      refill(slot);
    }
    if (++slot == stages) {
      slot = 0;
      parity ^= 1u;
    }
    cursor_step16<QT, M>(c, ntiles, nchunks, gc, g0);
  }
  return true;
}

// Lane 0, on an error path: waits (bounded) for the warp's `inflight` copies
// still landing in its ring, in slot order from (slot, parity), so that no
// bulk copy targets shared memory once the CTA has exited.
__device__ __forceinline__ void ring_drain(uint64_t* bars, int stages, int slot, uint32_t parity,
                                           int inflight) {
  for (int i = 0; i < inflight; ++i) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bars + slot, parity))
      if (clock64() - t0 > 4000000000LL) break;
    if (++slot == stages) {
      slot = 0;
      parity ^= 1u;
    }
  }
}

}  // namespace mlb

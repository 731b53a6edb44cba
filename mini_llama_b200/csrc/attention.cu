// attention.cu — split-K flash-decode attention over the fp32 KV cache.
//
// Reference: CudaAttentionDecodeDeviceInput (src/cuda_attention.cu:263-309:
// a score kernel writing [n_heads, pos+1] to global memory, then a per-head
// softmax + V-sum kernel, each followed by cudaDeviceSynchronize) and the CPU
// AttentionForward (src/forward.cc:487-545).
//
// Here one CTA handles one KV head and one slice of the positions [0, pos]:
// all q heads of the GQA group (h / (H/KV) == kv head) share each K/V tile,
// which is staged in shared memory with cp.async, scores and an online
// softmax (running max m, sum l) stay on chip, and the CTA writes (m, l, O)
// for its slice. The last CTA of a KV head to finish (arrival counter)
// combines the slices in slice order, so results are deterministic.
//
// include_current_v = 0 reproduces the reference CPU path (its V sum stops at
// t < pos while the softmax covers t <= pos, src/forward.cc:501-518);
// include_current_v = 1 is standard attention, as the reference GPU kernel.
#include <algorithm>
#include <cfloat>

#include <cuda_bf16.h>

#include "attention.cuh"

namespace mlb {

constexpr int kAttnThreads = 128;
constexpr int kAttnTile = 32;  // positions per shared-memory tile

struct AttnKArgs {
  const float* q;
  const float* keys;    // layer base [max_seq][KV][D]
  const float* values;
  const int* pos_dev;
  int pos_host;
  int H, KV, D, nsplit;
  float scale;
  int include_current_v;
  float* ws;            // [KV][nsplit][G][D + 2] per row
  int* counters;        // [KV] per row
  float* out;           // [H][D] per row
  // Batched form (grid.z = rows): row r reads q + r H D, writes out + r H D,
  // attends positions [0, row_pos[r]] of sequence row_seq[r] (row r when
  // null) whose cache starts seq_stride floats after the previous sequence's,
  // and uses the r-th workspace and counter block.
  const int* row_pos;
  const int* row_seq;
  long long seq_stride;
  int kv_bf16;
};

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnKArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int D = a.D, G = a.H / a.KV, KV = a.KV;
  const int pitch = D + 4;  // floats per staged row (no bank conflicts on 16-byte loads)
  const int kvh = blockIdx.x, split = blockIdx.y, row = blockIdx.z;
  const int seq = a.row_seq ? a.row_seq[row] : row;
  const float* keys = a.keys + (size_t)seq * a.seq_stride;
  const float* values = a.values + (size_t)seq * a.seq_stride;
  const float* qrow = a.q + (size_t)row * a.H * D;
  float* outrow = a.out + (size_t)row * a.H * D;
  float* wsrow = a.ws + (size_t)row * KV * a.nsplit * G * (D + 2);
  int* cnt = a.counters + (size_t)row * KV;
  float* kt = sm;                              // [2][tile][pitch]
  float* vt = kt + 2 * kAttnTile * pitch;      // [2][tile][pitch]
  const int hstep_ = kAttnThreads / (D / 4);
  const int region = max(4 * kAttnTile * pitch, hstep_ * G * D);  // K/V tiles, later group sums
  float* qs = sm + region;                     // [G][D]
  float* ps = qs + G * D;                      // [G][tile] probabilities
  float* part = ps + G * kAttnTile;            // [4 warps][G][tile] partial scores
  float* st = part + 4 * G * kAttnTile;        // [G] m, [G] l, [G] alpha
  float* mrun = st, *lrun = st + G, *alpha = st + 2 * G;
  __shared__ int last_flag;

  pdl_launch_dependents();  // dependents still wait for this grid to complete
  pdl_wait();
  const int pos = a.row_pos ? a.row_pos[row] : (a.pos_dev ? *a.pos_dev : a.pos_host);
  const int n = pos + 1;
  // slice of positions, in whole tiles
  const int tiles = (n + kAttnTile - 1) / kAttnTile;
  const int tiles_per = (tiles + a.nsplit - 1) / a.nsplit;
  const int t_begin = split * tiles_per * kAttnTile;
  const int t_end = min(n, (split + 1) * tiles_per * kAttnTile);
  const int v_end = a.include_current_v ? n : pos;  // V rows < v_end are summed

  for (int i = threadIdx.x; i < G * D; i += kAttnThreads)
    qs[i] = qrow[(size_t)(kvh * G) * D + i];
  for (int i = threadIdx.x; i < G; i += kAttnThreads) {
    mrun[i] = -INFINITY;
    lrun[i] = 0.0f;
  }
  const size_t row_stride = (size_t)KV * D;
  auto load_tile = [&](int t0, int buf) {
    const int vec = D / 4;
    for (int i = threadIdx.x; i < kAttnTile * vec; i += kAttnThreads) {
      int p = i / vec, c = i - p * vec;
      int t = t0 + p;
      float* kd = kt + (buf * kAttnTile + p) * pitch + c * 4;
      float* vd = vt + (buf * kAttnTile + p) * pitch + c * 4;
      if (t < t_end) {
        const size_t off = (size_t)t * row_stride + (size_t)kvh * D + c * 4;
        cp_async16(kd, keys + off);
        cp_async16(vd, values + off);
      } else {
        *reinterpret_cast<float4*>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    cp_async_commit();
  };

  // thread layout for scores: lane = position in tile, heads h = warp, warp+4, ...
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // thread layout for P.V: 4 consecutive d per thread; the hstep thread groups
  // split the positions of a tile and are summed once at the end (fixed order)
  const int dvec = D / 4;
  const int d4 = threadIdx.x % dvec, hg = threadIdx.x / dvec;
  const int hstep = kAttnThreads / dvec;
  const bool pv_active = hg < hstep;
  constexpr int kMaxG = 16;
  float4 o[kMaxG];
#pragma unroll
  for (int i = 0; i < kMaxG; ++i) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);

  if (t_begin < t_end) load_tile(t_begin, 0);
  __syncthreads();
  int buf = 0;
  for (int t0 = t_begin; t0 < t_end; t0 += kAttnTile, buf ^= 1) {
    if (t0 + kAttnTile < t_end) {
      load_tile(t0 + kAttnTile, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // scores: warp w takes a quarter of head_dim for every position (lane) and
    // every head of the group; the four partial dots are summed in warp order
    {
      const int nvec = D >> 2;
      const int v0 = warp * nvec / 4, v1 = (warp + 1) * nvec / 4;
      const float* krow = kt + (buf * kAttnTile + lane) * pitch;
      for (int h = 0; h < G; ++h) {
        const float* qh = qs + h * D;
        float dot = 0.0f;
        for (int vi = v0; vi < v1; ++vi) {
          const float4 kv = *reinterpret_cast<const float4*>(krow + vi * 4);
          const float4 qv = *reinterpret_cast<const float4*>(qh + vi * 4);
          dot = fmaf(qv.x, kv.x, dot);
          dot = fmaf(qv.y, kv.y, dot);
          dot = fmaf(qv.z, kv.z, dot);
          dot = fmaf(qv.w, kv.w, dot);
        }
        part[(warp * G + h) * kAttnTile + lane] = dot;
      }
    }
    __syncthreads();
    // per-head tile statistics and probabilities (warp per head)
    for (int h = warp; h < G; h += 4) {
      const float dot = ((part[(0 * G + h) * kAttnTile + lane] + part[(1 * G + h) * kAttnTile + lane]) +
                         part[(2 * G + h) * kAttnTile + lane]) + part[(3 * G + h) * kAttnTile + lane];
      const int t = t0 + lane;
      float s = t < t_end ? __fmul_rn(dot, a.scale) : -INFINITY;
      float tmax = warp_max(s);
      float mold = mrun[h];
      float mnew = fmaxf(mold, tmax);
      float p = t < t_end ? expf(s - mnew) : 0.0f;
      float psum = warp_sum(p);
      if (t >= v_end) p = 0.0f;  // softmax weight counted, V row not summed
      ps[h * kAttnTile + lane] = p;
      if (lane == 0) {
        float al = mold == -INFINITY ? 0.0f : expf(mold - mnew);
        alpha[h] = al;
        lrun[h] = lrun[h] * al + psum;
        mrun[h] = mnew;
      }
    }
    __syncthreads();
    // O = O * alpha + P . V  (this thread: d4, positions hg, hg + hstep, ...)
    const int tn = min(kAttnTile, t_end - t0);
    if (pv_active) {
#pragma unroll
      for (int h = 0; h < kMaxG; ++h) {
        if (h < G) {
          const float al = alpha[h];
          o[h].x *= al; o[h].y *= al; o[h].z *= al; o[h].w *= al;
        }
      }
      for (int p = hg; p < tn; p += hstep) {
        const float4 vv =
            *reinterpret_cast<const float4*>(vt + (buf * kAttnTile + p) * pitch + d4 * 4);
#pragma unroll
        for (int h = 0; h < kMaxG; ++h) {
          if (h < G) {
            const float pv = ps[h * kAttnTile + p];
            o[h].x = fmaf(pv, vv.x, o[h].x);
            o[h].y = fmaf(pv, vv.y, o[h].y);
            o[h].z = fmaf(pv, vv.z, o[h].z);
            o[h].w = fmaf(pv, vv.w, o[h].w);
          }
        }
      }
    }
    __syncthreads();
  }

  // sum the position groups (fixed order) through shared memory, then write
  // this slice's (m, l, O)
  float* gsum = kt;  // [hstep][G][D], reuses the K tiles
  if (pv_active) {
#pragma unroll
    for (int h = 0; h < kMaxG; ++h)
      if (h < G) *reinterpret_cast<float4*>(gsum + ((size_t)hg * G + h) * D + d4 * 4) = o[h];
  }
  __syncthreads();
  const int rec = D + 2;
  float* wsk = wsrow + ((size_t)kvh * a.nsplit + split) * G * rec;
  for (int i = threadIdx.x; i < G * D; i += kAttnThreads) {
    int h = i / D, d = i - h * D;
    float s = 0.0f;
    for (int gi = 0; gi < hstep; ++gi) s += gsum[((size_t)gi * G + h) * D + d];
    wsk[h * rec + 2 + d] = s;
  }
  for (int h = threadIdx.x; h < G; h += kAttnThreads) {
    wsk[h * rec] = mrun[h];
    wsk[h * rec + 1] = lrun[h];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_flag = atomicAdd(&cnt[kvh], 1) == a.nsplit - 1;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  // combine the slices of this KV head in slice order: per (head, slice) weight
  // e^(m_s - m) / l into shared memory, then every output element is one pass
  // of independent loads
  float* wsl = kt;  // [G][nsplit], reuses the K tiles (no cp.async in flight)
  for (int h = warp; h < G; h += 4) {
    float m = -INFINITY;
    for (int s = lane; s < a.nsplit; s += 32)
      m = fmaxf(m, __ldcg(wsrow + (((size_t)kvh * a.nsplit + s) * G + h) * rec));
    m = warp_max(m);
    float l = 0.0f;
    for (int s = lane; s < a.nsplit; s += 32) {
      const float* r = wsrow + (((size_t)kvh * a.nsplit + s) * G + h) * rec;
      const float ms = __ldcg(r);
      const float e = ms == -INFINITY ? 0.0f : expf(ms - m);
      wsl[h * a.nsplit + s] = e;
      l = fmaf(__ldcg(r + 1), e, l);
    }
    l = warp_sum(l);
    const float inv = 1.0f / l;
    __syncwarp();
    for (int s = lane; s < a.nsplit; s += 32) wsl[h * a.nsplit + s] *= inv;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += kAttnThreads) {
    const int h = i / D, d = i - h * D;
    const float* base = wsrow + ((size_t)kvh * a.nsplit * G + h) * rec + 2 + d;
    const size_t step = (size_t)G * rec;
    float acc = 0.0f;
    int s = 0;
    for (; s + 4 <= a.nsplit; s += 4) {
      const float o0 = __ldcg(base + (s + 0) * step), o1 = __ldcg(base + (s + 1) * step);
      const float o2 = __ldcg(base + (s + 2) * step), o3 = __ldcg(base + (s + 3) * step);
      acc = fmaf(o0, wsl[h * a.nsplit + s], acc);
      acc = fmaf(o1, wsl[h * a.nsplit + s + 1], acc);
      acc = fmaf(o2, wsl[h * a.nsplit + s + 2], acc);
      acc = fmaf(o3, wsl[h * a.nsplit + s + 3], acc);
    }
    for (; s < a.nsplit; ++s) acc = fmaf(__ldcg(base + s * step), wsl[h * a.nsplit + s], acc);
    outrow[(size_t)(kvh * G + h) * D + d] = acc;
  }
  if (threadIdx.x == 0) cnt[kvh] = 0;
}

// ------------------------------------------------------------ batched rows

constexpr int kRowsWarps = 8;
constexpr int kRowsThreads = kRowsWarps * 32;
// fp32 batched rows: blocks of PB positions in each warp's shared-memory ring
// (8 positions per warp, 64 KB per CTA at head_dim <= 128)
__host__ __device__ constexpr int rows_ring(int pb) { return 8 / pb; }
__host__ __device__ constexpr size_t rows_ring_bytes(int pb) {
  return (size_t)kRowsWarps * rows_ring(pb) * pb * 2 * 32 * 16;
}

// Sums NV values across the warp: afterwards v[0] of lane L holds the total of
// value index L / (32 / NV) (NV a power of two <= 32); each round keeps half
// of the remaining values and adds the partner lane's copy of that half.
template <int NV>
__device__ __forceinline__ void rows_multi_sum(float (&v)[NV], int lane) {
#pragma unroll
  for (int r = 0; r < 5; ++r) {
    const int off = 16 >> r;
    const int cnt = NV >> r;
    if (cnt > 1) {
      const int half = cnt >> 1;
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}

template <int G>
__device__ __forceinline__ void rows_combine(const AttnKArgs& a, float (&wm)[kRowsWarps][G],
                                             float (&wl)[kRowsWarps][G],
                                             float (&wo)[kRowsWarps][G][128],
                                             float (&cw)[G][kRowsWarps], int& last_flag, int kvh,
                                             int split, float* wsrow, float* outrow, int* cnt);

// Decode attention for batched rows: CTA (KV head, split, row) with 8 warps.
// Each warp streams blocks of PB positions of the split round robin, every
// lane holding 4 of the head_dim values of the K and V rows and of each
// query head of the GQA group (G heads, registers), and keeps an online
// softmax (m, l, o) per query head; the next block's rows are loaded before
// the current one is computed. The CTA then combines its 8 warps in warp
// order and, as in the tiled kernel, the last split of a head combines the
// splits in split order. head_dim is a multiple of 4 and at most 128.
// Four consecutive K or V elements of a row as fp32 (BF: stored as bf16,
// widened exactly).
template <int G, int PB, bool BF>
__global__ void __launch_bounds__(kRowsThreads, 2) attn_rows_kernel(const AttnKArgs a) {
  constexpr int NV = G * PB;
  static_assert(NV <= 32, "GQA group too large for one pass");
  constexpr unsigned kNvMask = NV >= 32 ? 0xffffffffu : ((1u << NV) - 1u);
  __shared__ float scw[kRowsWarps][NV];
  __shared__ float alw[kRowsWarps][G];
  __shared__ float wm[kRowsWarps][G], wl[kRowsWarps][G];
  __shared__ __align__(16) float wo[kRowsWarps][G][128];
  __shared__ float cw[G][kRowsWarps];
  __shared__ int last_flag;
  const int D = a.D, KV = a.KV;
  const int kvh = blockIdx.x, split = blockIdx.y, row = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();  // dependents still wait for this grid to complete
  pdl_wait();
  const int seq = a.row_seq ? a.row_seq[row] : row;
  const float* qrow = a.q + (size_t)row * a.H * D;
  float* outrow = a.out + (size_t)row * a.H * D;
  float* wsrow = a.ws + (size_t)row * KV * a.nsplit * G * (D + 2);
  int* cnt = a.counters + (size_t)row * KV;
  const int pos = a.row_pos ? a.row_pos[row] : (a.pos_dev ? *a.pos_dev : a.pos_host);
  const int n = pos + 1;
  const int v_end = a.include_current_v ? n : pos;
  // this split's positions, in whole warp blocks
  const int blocks = (n + PB - 1) / PB;
  const int per = (blocks + a.nsplit - 1) / a.nsplit;
  const int t_begin = min(n, split * per * PB), t_end = min(n, (split + 1) * per * PB);
  const bool dl = lane < (D >> 2);
  const size_t rstride = (size_t)KV * D;
  // this lane's 4 values in position 0's row of the sequence, and the bytes
  // from one position's row to the next
  constexpr size_t esz = BF ? 2 : 4;
  const size_t e0 = ((size_t)seq * a.seq_stride + (size_t)kvh * D + 4 * lane) * esz;
  const uint8_t* kb = reinterpret_cast<const uint8_t*>(a.keys) + e0;
  const uint8_t* vb = reinterpret_cast<const uint8_t*>(a.values) + e0;
  const size_t rbytes = rstride * esz;
  float4 q[G], o[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    q[h] = dl ? __ldg(reinterpret_cast<const float4*>(qrow + (size_t)(kvh * G + h) * D) + lane)
              : make_float4(0.f, 0.f, 0.f, 0.f);
    o[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float m_run = -INFINITY, l_run = 0.0f;  // lane i < NV: head i / PB
  // One warp block: the scores of positions tb .. tb + PB - 1 against every
  // query head of the group, the online softmax update and the V sum.
  auto block = [&](int tb, const float4 (&kx)[PB], const float4 (&vx)[PB]) {
    // the lane's 4-value dots as two paired partial sums (paired fp32
    // multiply and FMA: half the instructions of a scalar chain)
    float dv[NV];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        const float2 d = __ffma2_rn(make_float2(q[h].z, q[h].w), make_float2(kx[j].z, kx[j].w),
                                    __fmul2_rn(make_float2(q[h].x, q[h].y),
                                               make_float2(kx[j].x, kx[j].y)));
        dv[h * PB + j] = d.x + d.y;
      }
    rows_multi_sum<NV>(dv, lane);
    if ((lane & (32 / NV - 1)) == 0) scw[warp][lane / (32 / NV)] = dv[0];
    __syncwarp();
    if (lane < NV) {
      const int j = lane % PB;
      const int t = tb + j;
      const float sc = t < t_end ? __fmul_rn(scw[warp][lane], a.scale) : -INFINITY;
      float bmax = sc;
#pragma unroll
      for (int off = 1; off < PB; off <<= 1) bmax = fmaxf(bmax, __shfl_xor_sync(kNvMask, bmax, off));
      const float mnew = fmaxf(m_run, bmax);
      const float p = t < t_end ? expf(sc - mnew) : 0.0f;
      float psum = p;
#pragma unroll
      for (int off = 1; off < PB; off <<= 1) psum += __shfl_xor_sync(kNvMask, psum, off);
      const float al = m_run == -INFINITY ? 0.0f : expf(m_run - mnew);
      l_run = fmaf(l_run, al, psum);
      m_run = mnew;
      scw[warp][lane] = t < v_end ? p : 0.0f;  // counted in the softmax, V row summed below v_end
      if (j == 0) alw[warp][lane / PB] = al;
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < G; ++h) {
      // o = o * al + sum_j p_j v_j in paired fp32 operations (each pair
      // rounds as two scalar ones); o * 1 is o, so al == 1 skips the scaling
      const float al = alw[warp][h];  // the same in every lane
      float2 lo = make_float2(o[h].x, o[h].y), hi = make_float2(o[h].z, o[h].w);
      if (al != 1.0f) {
        lo = __fmul2_rn(lo, make_float2(al, al));
        hi = __fmul2_rn(hi, make_float2(al, al));
      }
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        const float p = scw[warp][h * PB + j];
        lo = __ffma2_rn(make_float2(p, p), make_float2(vx[j].x, vx[j].y), lo);
        hi = __ffma2_rn(make_float2(p, p), make_float2(vx[j].z, vx[j].w), hi);
      }
      o[h] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    __syncwarp();
  };
  const int tb0 = t_begin + warp * PB;
  constexpr int kStep = kRowsWarps * PB;  // from a warp's block to its next
  if constexpr (BF) {
    // bf16 rows: the next block's raw rows in registers while this one is
    // computed
    using Raw = KvRaw<BF>;
    using RawT = typename Raw::T;
    auto load_block = [&](int tb, RawT (&kx)[PB], RawT (&vx)[PB]) {
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        const int t = tb + j;
        kx[j] = (dl && t < t_end) ? Raw::load(kb + (size_t)t * rbytes) : Raw::zero();
        vx[j] = (dl && t < t_end && t < v_end) ? Raw::load(vb + (size_t)t * rbytes) : Raw::zero();
      }
    };
    RawT kn[PB], vn[PB];
    if (tb0 < t_end) load_block(tb0, kn, vn);
    for (int tb = tb0; tb < t_end; tb += kStep) {
      float4 kx[PB], vx[PB];
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        kx[j] = Raw::widen(kn[j]);
        vx[j] = Raw::widen(vn[j]);
      }
      if (tb + kStep < t_end) load_block(tb + kStep, kn, vn);
      block(tb, kx, vx);
    }
  } else {
    // fp32 rows: a ring of rows_ring(PB) blocks per warp in shared memory,
    // filled by cp.async, so all but one stay in flight during the arithmetic
    // without holding registers. Each lane copies and later reads only its
    // own 16 bytes of each row (no cross-lane ordering needed); a slot is
    // refilled at the end of its block, after its values were used.
    extern __shared__ uint4 kv_ring[];  // [warp][slot][j][K, V][lane]
    constexpr int R = rows_ring(PB);
    auto slot = [&](int r, int j, int kind) -> uint4* {
      return kv_ring + ((((size_t)warp * R + r) * PB + j) * 2 + kind) * 32 + lane;
    };
    auto issue = [&](int tb, int r) {
      if (dl) {
#pragma unroll
        for (int j = 0; j < PB; ++j) {
          const int t = tb + j;
          if (t < t_end) cp_async16(slot(r, j, 0), kb + (size_t)t * rbytes);
          if (t < t_end && t < v_end) cp_async16(slot(r, j, 1), vb + (size_t)t * rbytes);
        }
      }
      cp_async_commit();  // one group per block, empty past the split's end
    };
#pragma unroll
    for (int r = 0; r < R; ++r) issue(tb0 + r * kStep, r);
    int r = 0;
    for (int tb = tb0; tb < t_end; tb += kStep) {
      cp_async_wait<R - 1>();  // this block's group has landed
      float4 kx[PB], vx[PB];
#pragma unroll
      for (int j = 0; j < PB; ++j) {
        const int t = tb + j;
        const uint4 kr = *slot(r, j, 0), vr = *slot(r, j, 1);
        kx[j] = (dl && t < t_end) ? make_float4(__uint_as_float(kr.x), __uint_as_float(kr.y),
                                                __uint_as_float(kr.z), __uint_as_float(kr.w))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        vx[j] = (dl && t < t_end && t < v_end)
                    ? make_float4(__uint_as_float(vr.x), __uint_as_float(vr.y),
                                  __uint_as_float(vr.z), __uint_as_float(vr.w))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      block(tb, kx, vx);
      issue(tb + R * kStep, r);
      r = (r + 1) & (R - 1);
    }
    cp_async_wait<0>();
  }
  // this warp's (m, l, o) per query head
  if (lane < NV && lane % PB == 0) {
    wm[warp][lane / PB] = m_run;
    wl[warp][lane / PB] = l_run;
  }
  if (dl) {
#pragma unroll
    for (int h = 0; h < G; ++h) *reinterpret_cast<float4*>(&wo[warp][h][4 * lane]) = o[h];
  }
  rows_combine<G>(a, wm, wl, wo, cw, last_flag, kvh, split, wsrow, outrow, cnt);
}

// The end of both batched kernels, after every warp stored its (m, l, o) per
// query head (wm, wl, wo): the CTA's record with its warps combined in warp
// order, then, in the last split of the KV head to finish, the heads' outputs
// from the split records in split order.
template <int G>
__device__ __forceinline__ void rows_combine(const AttnKArgs& a, float (&wm)[kRowsWarps][G],
                                             float (&wl)[kRowsWarps][G],
                                             float (&wo)[kRowsWarps][G][128],
                                             float (&cw)[G][kRowsWarps], int& last_flag, int kvh,
                                             int split, float* wsrow, float* outrow, int* cnt) {
  const int D = a.D;
  __syncthreads();
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float m = -INFINITY;
    for (int w = 0; w < kRowsWarps; ++w) m = fmaxf(m, wm[w][h]);
    float l = 0.0f;
    for (int w = 0; w < kRowsWarps; ++w) {
      const float e = wm[w][h] == -INFINITY ? 0.0f : expf(wm[w][h] - m);
      cw[h][w] = e;
      l = fmaf(wl[w][h], e, l);
    }
    float* r = wsrow + (((size_t)kvh * a.nsplit + split) * G + h) * (D + 2);
    r[0] = m;
    r[1] = l;
  }
  __syncthreads();
  const int rec = D + 2;
  for (int i = threadIdx.x; i < G * D; i += kRowsThreads) {
    const int h = i / D, d = i - h * D;
    float acc = 0.0f;
    for (int w = 0; w < kRowsWarps; ++w) acc = fmaf(wo[w][h][d], cw[h][w], acc);
    wsrow[(((size_t)kvh * a.nsplit + split) * G + h) * rec + 2 + d] = acc;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_flag = atomicAdd(&cnt[kvh], 1) == a.nsplit - 1;
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  // the last split of the head combines the splits in split order
  float* wsl = &wo[0][0][0];  // [G][nsplit] weights (nsplit <= 8 * 128 / G)
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float m = -INFINITY;
    for (int s = 0; s < a.nsplit; ++s)
      m = fmaxf(m, __ldcg(wsrow + (((size_t)kvh * a.nsplit + s) * G + h) * rec));
    float l = 0.0f;
    for (int s = 0; s < a.nsplit; ++s) {
      const float* r = wsrow + (((size_t)kvh * a.nsplit + s) * G + h) * rec;
      const float ms = __ldcg(r);
      const float e = ms == -INFINITY ? 0.0f : expf(ms - m);
      wsl[h * a.nsplit + s] = e;
      l = fmaf(__ldcg(r + 1), e, l);
    }
    const float inv = 1.0f / l;
    for (int s = 0; s < a.nsplit; ++s) wsl[h * a.nsplit + s] *= inv;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += kRowsThreads) {
    const int h = i / D, d = i - h * D;
    float acc = 0.0f;
    for (int s = 0; s < a.nsplit; ++s)
      acc = fmaf(__ldcg(wsrow + (((size_t)kvh * a.nsplit + s) * G + h) * rec + 2 + d),
                 wsl[h * a.nsplit + s], acc);
    outrow[(size_t)(kvh * G + h) * D + d] = acc;
  }
  if (threadIdx.x == 0) cnt[kvh] = 0;
}

// A bf16 pair of two floats rounded to nearest even, x in the low half.
__device__ __forceinline__ uint32_t bf16x2_rn(float x, float y) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// hi = the bf16 pair of (x, y), lo = the bf16 pair of what hi leaves.
__device__ __forceinline__ void bf16x2_split(float x, float y, uint32_t& hi, uint32_t& lo) {
  hi = bf16x2_rn(x, y);
  lo = bf16x2_rn(x - __uint_as_float(hi << 16), y - __uint_as_float(hi & 0xffff0000u));
}

// D += A B, m16n8k16, bf16 operands, fp32 accumulators.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t u4_word(const uint4& v, int w) {
  return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
}

constexpr int kMmaD = 128;  // head_dim of the tensor-core kernel

// Tensor-core form of the batched kernel for a bf16 KV cache, head_dim 128 and
// G = 2, 4 or 8 query heads per KV head (mma.sync m16n8k16: bf16 operands,
// fp32 accumulators). A warp takes blocks of 16 positions of the split round
// robin:
//   S = Q K^T  A = the group's queries: row h holds head h rounded to bf16,
//              row 8 + h the bf16 rounding of what that leaves, so a score is
//              row h + row 8 + h of the accumulator (rows of heads past G are
//              zero); B = K, 8 positions per n-tile, two n-tiles, over the 8
//              chunks of 16 head_dim values.
//   O += P V   A = the probabilities split the same way, taken straight from
//              the score accumulators' registers; B = V, 16 positions by 8
//              head_dim columns, 16 n-tiles. The output is row h + row 8 + h.
// K and V values are exact bf16 operands, the hi/lo split keeps q and p to
// about 16 significant bits, and products are summed in fp32. Each lane reads
// 16 contiguous bytes of a K or V row per load: the head_dim order inside each
// 32 K values and the column order of the V n-tiles are permuted to match (q
// takes the same permutation; the output is stored in natural order). The
// online softmax per query head and the combines follow attn_rows_kernel.
template <int G>
__global__ void __launch_bounds__(kRowsThreads, 1) attn_rows_mma_kernel(const AttnKArgs a) {
  static_assert(G == 2 || G == 4 || G == 8, "GQA group of 2, 4 or 8 query heads");
  __shared__ float wm[kRowsWarps][G], wl[kRowsWarps][G];
  __shared__ __align__(16) float wo[kRowsWarps][G][128];
  __shared__ float cw[G][kRowsWarps];
  __shared__ uint4 qf[8][32];  // A fragments of the queries: [chunk][lane]
  __shared__ int last_flag;
  const int KV = a.KV;
  const int kvh = blockIdx.x, split = blockIdx.y, row = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  pdl_launch_dependents();  // dependents still wait for this grid to complete
  pdl_wait();
  const int seq = a.row_seq ? a.row_seq[row] : row;
  const float* qrow = a.q + (size_t)row * a.H * kMmaD;
  float* outrow = a.out + (size_t)row * a.H * kMmaD;
  float* wsrow = a.ws + (size_t)row * KV * a.nsplit * G * (kMmaD + 2);
  int* cnt = a.counters + (size_t)row * KV;
  const int pos = a.row_pos ? a.row_pos[row] : (a.pos_dev ? *a.pos_dev : a.pos_host);
  const int n = pos + 1;
  const int v_end = a.include_current_v ? n : pos;
  // this split's positions, in whole 16-position blocks
  const int blocks = (n + 15) / 16;
  const int per = (blocks + a.nsplit - 1) / a.nsplit;
  const int t_begin = min(n, split * per * 16), t_end = min(n, (split + 1) * per * 16);

  // Query fragments, thread i: chunk i / 32 of lane i % 32. Lane (g, t) of
  // chunk c holds head g's values 32 (c / 2) + 8 t + 4 (c % 2) + 0..3: the
  // first pair as k = 2t, 2t + 1 (a0 high part, a1 low part), the second as
  // k = 2t + 8, 2t + 9 (a2, a3).
  {
    const int c = threadIdx.x >> 5, lg = lane >> 2, lt = lane & 3;
    uint4 f = make_uint4(0u, 0u, 0u, 0u);
    if (lg < G) {
      const int v0 = (c >> 1) * 32 + lt * 8 + (c & 1) * 4;
      const float4 v =
          __ldg(reinterpret_cast<const float4*>(qrow + (size_t)(kvh * G + lg) * kMmaD + v0));
      bf16x2_split(v.x, v.y, f.x, f.y);
      bf16x2_split(v.z, v.w, f.z, f.w);
    }
    qf[c][lane] = f;
  }
  __syncthreads();

  const size_t rbytes = (size_t)KV * kMmaD * 2;  // from one position's row to the next
  const size_t e0 = ((size_t)seq * a.seq_stride + (size_t)kvh * kMmaD) * 2;
  const uint8_t* kb = reinterpret_cast<const uint8_t*>(a.keys) + e0 + tig * 16;
  const uint8_t* vb = reinterpret_cast<const uint8_t*>(a.values) + e0 + g * 16;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;  // head g; l_run: this lane's positions only
  // K of block tb, n-tile nt: position tb + 8 nt + g, values 32 cp + 8 t .. + 7
  uint4 kr[2][4];
  auto load_k = [&](int tb) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int t = tb + 8 * nt + g;
      const uint8_t* p = kb + (size_t)t * rbytes;
#pragma unroll
      for (int cp = 0; cp < 4; ++cp)
        kr[nt][cp] = t < t_end ? __ldcs(reinterpret_cast<const uint4*>(p + cp * 64)) : z4;
    }
  };
  // V of block tb: positions tb + 2 t + {0, 1, 8, 9}, columns 64 s + 8 g .. + 7
  uint4 vr[2][4];
  auto load_v = [&](int tb) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = tb + 2 * tig + (r & 1) + 8 * (r >> 1);
      const uint8_t* p = vb + (size_t)t * rbytes;
      const bool in = t < t_end && t < v_end;
#pragma unroll
      for (int s = 0; s < 2; ++s)
        vr[s][r] = in ? __ldcs(reinterpret_cast<const uint4*>(p + s * 128)) : z4;
    }
  };
  // The next block's K is loaded once the scores have used this block's, and
  // its V once P V has used this block's, so loads stay in flight across the
  // arithmetic without more registers.
  const int tb0 = t_begin + warp * 16;
  if (tb0 < t_end) {
    load_k(tb0);
    load_v(tb0);
  }
  for (int tb = tb0; tb < t_end; tb += kRowsWarps * 16) {
    const int tn = tb + kRowsWarps * 16;  // the warp's next block
    // scores of head g at positions tb + 8 nt + 2 t + e: acc[nt][e] + acc[nt][2 + e]
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 f = qf[c][lane];
      const uint32_t A[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const uint4& k = kr[nt][c >> 1];
        mma_bf16_16816(sacc[nt], A, (c & 1) ? k.z : k.x, (c & 1) ? k.w : k.y);
      }
    }
    if (tn < t_end) load_k(tn);
    float sc[2][2];
    float bmax = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tb + 8 * nt + 2 * tig + e;
        sc[nt][e] = t < t_end ? __fmul_rn(sacc[nt][e] + sacc[nt][2 + e], a.scale) : -INFINITY;
        bmax = fmaxf(bmax, sc[nt][e]);
      }
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
    bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
    const float mnew = fmaxf(m_run, bmax);
    const float al = m_run == -INFINITY ? 0.0f : expf(m_run - mnew);
    float psum = 0.0f, pv[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tb + 8 * nt + 2 * tig + e;
        const float p = t < t_end ? expf(sc[nt][e] - mnew) : 0.0f;
        psum += p;
        pv[nt][e] = t < v_end ? p : 0.0f;  // counted in the softmax, V row summed below v_end
      }
    l_run = fmaf(l_run, al, psum);
    m_run = mnew;
    if (__any_sync(0xffffffffu, al != 1.0f)) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[j][i] *= al;
    }
    // A = P: rows g / 8 + g the high / low parts, k = 2 t + e (n-tile 0) and
    // 2 t + 8 + e (n-tile 1)
    uint32_t P[4];
    bf16x2_split(pv[0][0], pv[0][1], P[0], P[1]);
    bf16x2_split(pv[1][0], pv[1][1], P[2], P[3]);
    // n-tile 8 s + e, column g: value 64 s + 8 g + e; k pairs (2 t, 2 t + 1)
    // and (2 t + 8, 2 t + 9) from two positions' words
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t sel = (e & 1) ? 0x7632u : 0x5410u;
        const uint32_t b0 = __byte_perm(u4_word(vr[s][0], e >> 1), u4_word(vr[s][1], e >> 1), sel);
        const uint32_t b1 = __byte_perm(u4_word(vr[s][2], e >> 1), u4_word(vr[s][3], e >> 1), sel);
        mma_bf16_16816(o[8 * s + e], P, b0, b1);
      }
    if (tn < t_end) load_v(tn);
  }
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (g < G) {
    if (tig == 0) {
      wm[warp][g] = m_run;
      wl[warp][g] = l_run;
    }
    // accumulator columns 2 t, 2 t + 1 of n-tile 8 s + e: values 64 s + 8 (2 t) + e, + 8
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = 8 * s + e;
        wo[warp][g][64 * s + 16 * tig + e] = o[j][0] + o[j][2];
        wo[warp][g][64 * s + 16 * tig + 8 + e] = o[j][1] + o[j][3];
      }
  }
  rows_combine<G>(a, wm, wl, wo, cw, last_flag, kvh, split, wsrow, outrow, cnt);
}

// Generic path for shapes the tiled kernel does not take (head_dim not a
// multiple of 4, or more than 16 query heads per KV head): one CTA per query
// head, scores in shared memory, one pass per output element.
__global__ void attn_decode_generic_kernel(const AttnKArgs a) {
  extern __shared__ float sc[];  // [pos + 1]
  __shared__ float red[32];
  __shared__ float bc;
  const int h = blockIdx.x, G = a.H / a.KV, kvh = h / G, D = a.D;
  const int pos = a.pos_dev ? *a.pos_dev : a.pos_host;
  const int n = pos + 1, v_end = a.include_current_v ? n : pos;
  const size_t stride = (size_t)a.KV * D;
  const float* qh = a.q + (size_t)h * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float m = -INFINITY;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float* k = a.keys + (size_t)t * stride + (size_t)kvh * D;
    float dot = 0.0f;
    for (int d = 0; d < D; ++d) dot = fmaf(qh[d], k[d], dot);
    float s = __fmul_rn(dot, a.scale);
    sc[t] = s;
    m = fmaxf(m, s);
  }
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int i = 1; i < nw; ++i) t = fmaxf(t, red[i]);
    bc = t;
  }
  __syncthreads();
  m = bc;
  float l = 0.0f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    float e = expf(sc[t] - m);
    sc[t] = e;
    l += e;
  }
  l = warp_sum(l);
  __syncthreads();
  if (lane == 0) red[warp] = l;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += red[i];
    bc = t;
  }
  __syncthreads();
  l = bc;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.0f;
    for (int t = 0; t < v_end; ++t)
      acc = fmaf(sc[t], a.values[(size_t)t * stride + (size_t)kvh * D + d], acc);
    a.out[(size_t)h * D + d] = __fdiv_rn(acc, l);
  }
}

bool attn_tiled_ok(int H, int KV, int D) {
  return D % 4 == 0 && D <= 512 && H / KV <= 16 && attn_smem_bytes(H / KV, D) <= 200 * 1024;
}

size_t attn_smem_bytes(int G, int D) {
  const int pitch = D + 4;
  const int hstep = kAttnThreads / (D / 4);
  const int region = std::max(4 * kAttnTile * pitch, hstep * G * D);
  return (size_t)(region + G * D + 5 * G * kAttnTile + 3 * G) * sizeof(float);
}

int attn_splits(int KV, int sms, int max_seq) {
  int tiles = (max_seq + kAttnTile - 1) / kAttnTile;
  int want = (3 * sms + KV - 1) / KV;
  int s = want < tiles ? want : tiles;
  return s < 1 ? 1 : s;
}

void attn_check(int H, int KV, int D) {
  if (H <= 0 || KV <= 0 || D <= 0) invalid("attention: head counts and head_dim must be positive");
  if (H % KV != 0) invalid("attention: n_heads must be divisible by n_kv_heads");
}

void attn_check_tiled(int H, int KV, int D) {
  attn_check(H, KV, D);
  if (!attn_tiled_ok(H, KV, D))
    invalid("decode step: head_dim must be a multiple of 4 (<= 512) with <= 16 query heads per "
            "KV head");
}

void attn_launch(const AttnLaunch& l, cudaStream_t stream, bool pdl) {
  AttnKArgs a;
  a.q = l.q;
  a.keys = l.keys;
  a.values = l.values;
  a.pos_dev = l.pos_dev;
  a.pos_host = l.pos_host;
  a.H = l.H;
  a.KV = l.KV;
  a.D = l.D;
  a.nsplit = l.nsplit;
  a.scale = l.scale;
  a.include_current_v = l.include_current_v;
  a.ws = l.ws;
  a.counters = l.counters;
  a.out = l.out;
  a.row_pos = l.row_pos;
  a.row_seq = l.row_seq;
  a.seq_stride = l.seq_stride;
  a.kv_bf16 = l.kv_bf16;
  int dev = 0;
  MLB_CUDA(cudaGetDevice(&dev));
  if (l.rows < 1) invalid("attention: no rows");
  if (!attn_tiled_ok(l.H, l.KV, l.D)) {
    if (l.rows != 1 || l.row_pos) invalid("attention: batched rows need the tiled kernel");
    const int pos = l.pos_host;
    if (l.pos_dev) invalid("attention: the generic path takes a host position");
    const size_t gsm = (size_t)(pos + 1) * sizeof(float);
    if (gsm > 200 * 1024) invalid("attention: position too large for this head shape");
    if (gsm > 48 * 1024)
      MLB_CUDA(cudaFuncSetAttribute(attn_decode_generic_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gsm));
    launch_pdl(attn_decode_generic_kernel, dim3(l.H), dim3(kAttnThreads), gsm, stream, pdl, a);
    return;
  }
  const int G = l.H / l.KV;
  const bool rows_ok = l.D % 4 == 0 && l.D <= 128 && (G == 1 || G == 2 || G == 4 || G == 8);
  if (l.kv_bf16 && (!l.row_pos || !rows_ok))
    invalid("attention: a bf16 KV cache needs batched rows, head_dim a multiple of 4 up to 128 "
            "and 1, 2, 4 or 8 query heads per KV head");
  if (l.row_pos && rows_ok) {
    // batched rows: the register-streaming kernel (its combine keeps G x
    // nsplit split weights in 8 x G x 128 floats)
    a.nsplit = std::max(1, std::min(l.nsplit, kRowsWarps * 128));
    const dim3 grid(l.KV, a.nsplit, l.rows);
    if (l.kv_bf16 && l.D == kMmaD && G >= 2) {
      // bf16 K/V, head_dim 128: the tensor-core kernel
      switch (G) {
        case 2: launch_pdl(attn_rows_mma_kernel<2>, grid, dim3(kRowsThreads), 0, stream, pdl, a); break;
        case 4: launch_pdl(attn_rows_mma_kernel<4>, grid, dim3(kRowsThreads), 0, stream, pdl, a); break;
        default: launch_pdl(attn_rows_mma_kernel<8>, grid, dim3(kRowsThreads), 0, stream, pdl, a); break;
      }
      return;
    }
    auto go = [&](auto f32_kernel, auto bf16_kernel, int pb, int gi) {
      if (l.kv_bf16) {
        launch_pdl(bf16_kernel, grid, dim3(kRowsThreads), 0, stream, pdl, a);
      } else {
        // the fp32 kernel's K/V ring: dynamic shared memory above 48 KB
        const size_t ring = rows_ring_bytes(pb);
        static bool set[64][4] = {};
        if (dev < 64 && !set[dev][gi]) {
          MLB_CUDA(cudaFuncSetAttribute(f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)ring));
          set[dev][gi] = true;
        }
        launch_pdl(f32_kernel, grid, dim3(kRowsThreads), ring, stream, pdl, a);
      }
    };
    switch (G) {
      case 1: go(attn_rows_kernel<1, 4, false>, attn_rows_kernel<1, 4, true>, 4, 0); break;
      case 2: go(attn_rows_kernel<2, 4, false>, attn_rows_kernel<2, 4, true>, 4, 1); break;
      case 4: go(attn_rows_kernel<4, 4, false>, attn_rows_kernel<4, 4, true>, 4, 2); break;
      default: go(attn_rows_kernel<8, 2, false>, attn_rows_kernel<8, 2, true>, 2, 3); break;
    }
    return;
  }
  {
    // the combine keeps G x nsplit slice weights in the K/V tile region
    const int pitch = l.D + 4, hstep = kAttnThreads / (l.D / 4);
    const int region = std::max(4 * kAttnTile * pitch, hstep * G * l.D);
    a.nsplit = std::max(1, std::min(l.nsplit, region / G));
  }
  const size_t smem = attn_smem_bytes(l.H / l.KV, l.D);
  static size_t smem_set[64] = {};
  if (dev < 64 && smem > 48 * 1024 && smem_set[dev] < smem) {
    MLB_CUDA(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    smem_set[dev] = smem;
  }
  launch_pdl(attn_decode_kernel, dim3(l.KV, a.nsplit, l.rows), dim3(kAttnThreads), smem, stream,
             pdl, a);
}

size_t attn_ws_floats(int H, int KV, int D, int nsplit) {
  return (size_t)KV * nsplit * (H / KV) * (D + 2);
}

}  // namespace mlb

// sample.cu — MiniSampler::Sample (src/sampler.cc:107-183) on the device.
//
// One CTA of 1024 threads per sample. The steps follow the reference:
//   * every logit must be finite (ValidateLogits, src/sampler.cc:16-25);
//   * temperature < 1e-6 or top_k == 1: greedy, the first index of the
//     maximum (ArgMax, src/ops.cc:220-233), and no random draw;
//   * top_k > 1: the top_k largest logits (ties: lower index first,
//     src/sampler.cc:160-165), in that order, are the candidates;
//     top_k == 0: every logit, in index order;
//   * p_i = exp((x_i - max) / T), r = one uniform float from the sampler's
//     std::mt19937 (uniform_real_distribution<float>(0, 1), which takes one
//     32-bit word: r = float(u) * 2^-32, kept below 1), and the first
//     candidate whose running sum of p_i / sum exceeds r is the sample; the
//     last candidate when none does (src/sampler.cc:45-87).
// The generator is the published MT19937 (Matsumoto & Nishimura, 1998), the
// algorithm std::mt19937 specifies, so the draws equal the reference's word
// for word. The sums run as fixed-order block reductions rather than one
// sequential loop, and exp is CUDA's expf: the sample equals the reference's
// except when r falls within rounding distance of a candidate boundary.
//
// Top-k selection: a most-significant-byte-first radix select over the
// order-preserving 32-bit key of each logit (four passes, per-warp byte
// histograms in shared memory) finds the k-th largest key; the keys above it
// and the first ones equal to it in index order are gathered and sorted
// (bitonic, descending by value then ascending index).
#include <algorithm>

#include "gemv.cuh"
#include "sample.cuh"

namespace mlb {

namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr float kGreedyTemperature = 1e-6f;  // src/sampler.cc:13

// ---------------------------------------------------------------- MT19937

__device__ uint32_t mt_draw(MtState* st) {
  if (st->idx >= kMtN) {
    for (int k = 0; k < kMtN; ++k) {
      const uint32_t y = (st->mt[k] & 0x80000000u) | (st->mt[(k + 1) % kMtN] & 0x7fffffffu);
      st->mt[k] = st->mt[(k + 397) % kMtN] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
    }
    st->idx = 0;
  }
  uint32_t y = st->mt[st->idx++];
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

// uniform_real_distribution<float>(0, 1) over one word: float(u) / 2^32,
// and the largest float below 1 when that rounds up to 1.
__device__ float mt_uniform(MtState* st) {
  const float r = __uint2float_rn(mt_draw(st)) * 2.3283064365386963e-10f;  // 2^-32, exact
  return r >= 1.0f ? __uint_as_float(0x3F7FFFFFu) : r;
}

// ------------------------------------------------------- block primitives

__device__ __forceinline__ unsigned int key_hi(unsigned long long k) {
  return (unsigned int)(k >> 32);
}
// The logit a key encodes (finite values only).
__device__ __forceinline__ float key_value(unsigned long long k) {
  const unsigned int u = key_hi(k);
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
__device__ __forceinline__ int key_index(unsigned long long k) { return argmax_index_of(k); }

// Exclusive prefix sum of one int per thread, in thread order.
__device__ int block_excl_scan(int v, int* sw) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sw[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = sw[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    sw[lane] = t;  // inclusive warp totals
  }
  __syncthreads();
  const int r = (warp ? sw[warp - 1] : 0) + x - v;
  __syncthreads();
  return r;
}

// Exclusive prefix sum of one float per thread, in thread order (fixed
// association: within a warp by the shuffle ladder, then warp totals).
__device__ float block_excl_scan_f(float v, float* sw) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sw[warp] = x;
  __syncthreads();
  if (warp == 0) {
    float t = sw[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    sw[lane] = t;
  }
  __syncthreads();
  float e = __shfl_up_sync(0xffffffffu, x, 1);  // the lanes before this one
  if (lane == 0) e = 0.0f;
  const float r = (warp ? sw[warp - 1] : 0.0f) + e;
  __syncthreads();
  return r;
}

// Sum of one float per thread in a fixed tree order; every thread gets it.
__device__ float block_sum_f(float v, float* sw) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) sw[warp] = v;
  __syncthreads();
  float t = lane < kSampleWarps ? sw[lane] : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  __syncthreads();
  return t;
}

__device__ int block_min_i(int v, int* sw) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) sw[warp] = v;
  __syncthreads();
  int t = lane < kSampleWarps ? sw[lane] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = min(t, __shfl_xor_sync(0xffffffffu, t, o));
  __syncthreads();
  return t;
}

// Every thread visits i = tid, tid + 1024, ... < n, loading 8 of its values
// before using any (one CTA streams the whole row several times, so each
// thread keeps several loads in flight). f(v, i, valid) is called by every
// lane of a warp the same number of times (valid false past n), so it may
// use warp-wide primitives.
constexpr int kBatch = 8;
template <class F>
__device__ __forceinline__ void for_strided(const float* __restrict__ x, int n, F f) {
  for (int base = threadIdx.x - (threadIdx.x & 31); base < n; base += kBatch * kSampleThreads) {
    float v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = base + j * kSampleThreads + (threadIdx.x & 31);
      v[j] = i < n ? __ldcg(x + i) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = base + j * kSampleThreads + (threadIdx.x & 31);
      f(v[j], i, i < n);
    }
  }
}
// The same over this thread's contiguous range [lo, hi), in index order.
template <class F>
__device__ __forceinline__ void for_range(const float* __restrict__ x, int lo, int hi, F f) {
  for (int base = lo; base < hi; base += kBatch) {
    float v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) v[j] = base + j < hi ? __ldcg(x + base + j) : 0.0f;
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (base + j < hi) f(v[j], base + j);
  }
}

// ------------------------------------------------------------------ kernel

__global__ void __launch_bounds__(kSampleThreads, 1)
    sample_kernel(const float* __restrict__ logits, int n, float temperature, int top_k,
                  MtState* st, int* out_id, DeviceStatus* status, int* token, int* tokens,
                  const int* step) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ float s_f[kSampleWarps];
  __shared__ int s_i[kSampleWarps];
  __shared__ unsigned long long s_k[kSampleWarps];
  __shared__ unsigned int s_tot[256];
  __shared__ unsigned int s_prefix, s_mask;
  __shared__ int s_rem, s_cnt;
  __shared__ float s_r;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // finiteness, the maximum and the greedy key
  float mx = -INFINITY;
  unsigned long long best = 0ull;
  int bad = 0;
  for_strided(logits, n, [&](float v, int i, bool valid) {
    if (!valid) return;
    if (!isfinite(v)) {
      bad = 1;
      return;
    }
    mx = fmaxf(mx, v);
    const unsigned long long k = argmax_key_of(v, i);
    best = k > best ? k : best;
  });
  bad = __syncthreads_or(bad);
  if (bad) {
    if (tid == 0 && atomicCAS(&status->code, 0, MLB_ERR_INVALID) == 0)
      atomicExch(&status->where, 700);
    return;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  best = warp_max_u64(best);
  if (lane == 0) {
    s_f[warp] = mx;
    s_k[warp] = best;
  }
  __syncthreads();
  if (warp == 0) {
    float m = lane < kSampleWarps ? s_f[lane] : -INFINITY;
    unsigned long long b = lane < kSampleWarps ? s_k[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    b = warp_max_u64(b);
    if (lane == 0) {
      s_f[0] = m;
      s_k[0] = b;
    }
  }
  __syncthreads();
  mx = s_f[0];
  best = s_k[0];
  __syncthreads();

  int id;
  if (temperature < kGreedyTemperature || top_k == 1) {
    id = argmax_index_of(best);
  } else {
    if (tid == 0) s_r = mt_uniform(st);
    __syncthreads();
    const float r = s_r;
    if (top_k > 1) {
      const int kk = min(top_k, n);
      // radix select of the kk-th largest key
      unsigned int* hist = reinterpret_cast<unsigned int*>(dyn);  // [warps][256]
      if (tid == 0) {
        s_prefix = 0u;
        s_mask = 0u;
        s_rem = kk;
      }
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int j = tid; j < kSampleWarps * 256; j += kSampleThreads) hist[j] = 0u;
        __syncthreads();
        const unsigned int prefix = s_prefix, mask = s_mask;
        // lanes of a warp that fall in the same bin add once (logits crowd
        // into a few bins of the leading bytes)
        for_strided(logits, n, [&](float v, int i, bool valid) {
          const unsigned int u = valid ? key_hi(argmax_key_of(v, i)) : 0u;
          const bool act = valid && (u & mask) == prefix;
          const unsigned int am = __ballot_sync(0xffffffffu, act);
          if (act) {
            const unsigned int bin = (u >> shift) & 255u;
            const unsigned int peers = __match_any_sync(am, bin);
            if (lane == __ffs(peers) - 1) atomicAdd(&hist[warp * 256 + bin], __popc(peers));
          }
        });
        __syncthreads();
        if (tid < 256) {
          unsigned int t = 0;
          for (int w = 0; w < kSampleWarps; ++w) t += hist[w * 256 + tid];
          s_tot[tid] = t;
        }
        __syncthreads();
        if (tid == 0) {
          int cum = 0;
          for (int b = 255; b >= 0; --b) {
            if (cum + (int)s_tot[b] >= s_rem) {
              s_prefix |= (unsigned int)b << shift;
              s_mask |= 255u << shift;
              s_rem -= cum;
              break;
            }
            cum += (int)s_tot[b];
          }
        }
        __syncthreads();
      }
      const unsigned int thr = s_prefix;
      const int need_eq = s_rem, cnt_gt = kk - s_rem;
      int kp = 2;
      while (kp < kk) kp <<= 1;
      unsigned long long* cand = reinterpret_cast<unsigned long long*>(dyn);  // [kp]
      if (tid == 0) s_cnt = 0;
      __syncthreads();
      for_strided(logits, n, [&](float v, int i, bool valid) {
        const unsigned long long k = argmax_key_of(v, i);
        if (valid && key_hi(k) > thr) cand[atomicAdd(&s_cnt, 1)] = k;
      });
      // the keys equal to the threshold: the first need_eq in index order
      const int chunk = (n + kSampleThreads - 1) / kSampleThreads;
      const int lo = min(n, tid * chunk), hi = min(n, lo + chunk);
      int c = 0;
      for_range(logits, lo, hi,
                [&](float v, int i) { c += key_hi(argmax_key_of(v, i)) == thr; });
      int base = block_excl_scan(c, s_i);
      if (c > 0 && base < need_eq)
        for_range(logits, lo, hi, [&](float v, int i) {
          const unsigned long long k = argmax_key_of(v, i);
          if (key_hi(k) == thr && base < need_eq) cand[cnt_gt + base++] = k;
        });
      for (int j = kk + tid; j < kp; j += kSampleThreads) cand[j] = 0ull;
      __syncthreads();
      // bitonic sort, descending
      for (int size = 2; size <= kp; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int t = tid; t < kp / 2; t += kSampleThreads) {
            const int i = 2 * stride * (t / stride) + (t % stride), j = i + stride;
            const unsigned long long a = cand[i], b = cand[j];
            const bool desc = (i & size) == 0;
            if ((a < b) == desc) {
              cand[i] = b;
              cand[j] = a;
            }
          }
          __syncthreads();
        }
      }
      // softmax weights of the candidates in sorted order; thread t holds
      // candidates 4t .. 4t + 3
      const float m = key_value(cand[0]);
      float p[4];
      float ls = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = 4 * tid + q;
        p[q] = j < kk ? expf(__fdiv_rn(__fsub_rn(key_value(cand[j]), m), temperature)) : 0.0f;
        ls += p[q];
      }
      const float sum = block_sum_f(ls, s_f);
      float lq = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        p[q] = __fdiv_rn(p[q], sum);
        lq += p[q];
      }
      float cum = block_excl_scan_f(lq, s_f);
      int found = 0x7fffffff;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = 4 * tid + q;
        cum += p[q];
        if (j < kk && found == 0x7fffffff && r < cum) found = j;
      }
      found = block_min_i(found, s_i);
      id = key_index(cand[found == 0x7fffffff ? kk - 1 : found]);
    } else {
      // every logit in index order; thread t holds the contiguous range
      // [t chunk, (t + 1) chunk)
      const int chunk = (n + kSampleThreads - 1) / kSampleThreads;
      const int lo = min(n, tid * chunk), hi = min(n, lo + chunk);
      auto weight = [&](float v) { return expf(__fdiv_rn(__fsub_rn(v, mx), temperature)); };
      float ls = 0.0f;
      for_range(logits, lo, hi, [&](float v, int) { ls += weight(v); });
      const float sum = block_sum_f(ls, s_f);
      float lq = 0.0f;
      for_range(logits, lo, hi, [&](float v, int) { lq += __fdiv_rn(weight(v), sum); });
      float cum = block_excl_scan_f(lq, s_f);
      int found = 0x7fffffff;
      // the running sum at element i is cum + (this thread's sum up to i,
      // added from 0 as for lq), so only a thread with r < cum + lq holds
      // the crossing
      if (r < cum + lq) {
        float part = 0.0f;
        for_range(logits, lo, hi, [&](float v, int i) {
          part += __fdiv_rn(weight(v), sum);
          if (found == 0x7fffffff && r < cum + part) found = i;
        });
      }
      found = block_min_i(found, s_i);
      id = found == 0x7fffffff ? n - 1 : found;
    }
  }
  if (tid == 0) {
    *out_id = id;
    if (token) {
      *token = id;
      tokens[*step - 1] = id;
    }
  }
}

}  // namespace

void mt_seed(uint32_t seed, MtState* out) {
  out->mt[0] = seed;
  for (int i = 1; i < kMtN; ++i)
    out->mt[i] = 1812433253u * (out->mt[i - 1] ^ (out->mt[i - 1] >> 30)) + (uint32_t)i;
  out->idx = kMtN;
}

void sample_launch(const float* logits, int n, float temperature, int top_k, MtState* st,
                   int* out_id, DeviceStatus* status, int* token, int* tokens, const int* step,
                   cudaStream_t stream) {
  const size_t smem = std::max<size_t>((size_t)kSampleWarps * 256 * 4, (size_t)kSampleMaxTopK * 8);
  sample_kernel<<<1, kSampleThreads, smem, stream>>>(logits, n, temperature, top_k, st, out_id,
                                                      status, token, tokens, step);
  MLB_CUDA(cudaGetLastError());
}

}  // namespace mlb

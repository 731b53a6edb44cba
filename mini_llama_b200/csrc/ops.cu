// ops.cu — small device ops: the standalone elementwise entry points, KV-cache
// write, embedding row, argmax, RoPE tables and the seeded weight generator.
//
// References: RMSNorm / SiLU / Mul / Add / Softmax / Embedding / RoPE kernels
// of src/cuda_ops.cu:28-206 and their CPU definitions in src/ops.cc:43-233;
// the KV write of CudaKvCache::WriteDevice (src/cuda_kv_cache.cc:137-163).
// Arithmetic that the CPU path rounds step by step is written with _rn
// intrinsics so no multiply-add is fused where the CPU rounds twice.
#include <cmath>
#include <vector>

#include "gemv.cuh"
#include "ops.cuh"
#include "synth.h"

namespace mlb {

// ------------------------------------------------------------ elementwise

// One CTA: y = (x * 1/sqrt(mean(x^2) + eps)) * w, deterministic tree sum.
__global__ void rmsnorm_kernel(const float* x, const float* w, int n, float eps, float* y) {
  __shared__ float part[32];
  __shared__ float scale;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += part[i];
    scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(t, (float)n), eps)));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fmul_rn(__fmul_rn(x[i], scale), w[i]);
}

__global__ void silu_kernel(const float* x, int n, float* y) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    float v = x[i];
    y[i] = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));  // x / (1 + e^-x), src/ops.cc:106
  }
}
__global__ void mul_kernel(const float* a, const float* b, int n, float* y) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fmul_rn(a[i], b[i]);
}
__global__ void add_kernel(const float* a, const float* b, int n, float* y) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

// One CTA softmax (src/ops.cc:71-98).
__global__ void softmax_kernel(const float* x, int n, float* y) {
  __shared__ float part[32];
  __shared__ float bc;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
  m = warp_max(m);
  if (lane == 0) part[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = part[0];
    for (int i = 1; i < nw; ++i) t = fmaxf(t, part[i]);
    bc = t;
  }
  __syncthreads();
  m = bc;
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float e = expf(x[i] - m);
    y[i] = e;
    s += e;
  }
  s = warp_sum(s);
  __syncthreads();
  if (lane == 0) part[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += part[i];
    bc = t;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[i] = __fdiv_rn(y[i], bc);
}

// Embedding row; the token comes from the host or from device memory.
__global__ void embedding_kernel(const float* table, int vocab, int dim, const int* token_dev,
                                 int token_host, float* y) {
  pdl_launch_dependents();
  pdl_wait();
  int tok = token_dev ? *token_dev : token_host;
  if (tok < 0 || tok >= vocab) return;  // validated on the host before launch
  const float* row = table + (size_t)tok * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    y[i] = row[i];
}

// RoPE on q [nh, D] and k [nkv, D] with precomputed (cos, sin) per pair index.
__global__ void rope_kernel(float* q, float* k, int nh, int nkv, int D, int neox,
                            const float2* cs) {
  int half = D / 2;
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  int total = (nh + nkv) * half;
  if (i >= total) return;
  int head = i / half, j = i - head * half;
  float* v = head < nh ? q + (size_t)head * D : k + (size_t)(head - nh) * D;
  int i0 = neox ? j : 2 * j, i1 = neox ? j + half : 2 * j + 1;
  float a = v[i0], b = v[i1];
  float2 c = cs[j];
  v[i0] = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
  v[i1] = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
}

__global__ void kv_write_kernel(float* keys, float* values, size_t slot, int n, const float* k,
                                const float* v) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    keys[slot + i] = k[i];
    values[slot + i] = v[i];
  }
}

// Argmax with the lowest index winning ties (src/ops.cc:220-233). One CTA;
// writes the index to out_dev and optionally to a second slot.
__global__ void argmax_kernel(const float* x, int n, int* out_dev, int* out_dev2) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  pdl_wait();
  pdl_launch_dependents();
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = x[i];
    if (v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
        best = bv[w];
        idx = bi[w];
      }
    if (idx == 0x7fffffff) idx = 0;  // all NaN: the reference keeps index 0
    *out_dev = idx;
    if (out_dev2) *out_dev2 = idx;
  }
}

// ------------------------------------------------------------- launchers

static unsigned blocks_for(long long n, int t = 256) { return (unsigned)((n + t - 1) / t); }

void op_rmsnorm(const float* x, const float* w, int n, float eps, float* y, cudaStream_t s) {
  rmsnorm_kernel<<<1, 1024, 0, s>>>(x, w, n, eps, y);
  MLB_CUDA(cudaGetLastError());
}
void op_silu(const float* x, int n, float* y, cudaStream_t s) {
  silu_kernel<<<blocks_for(n), 256, 0, s>>>(x, n, y);
  MLB_CUDA(cudaGetLastError());
}
void op_mul(const float* a, const float* b, int n, float* y, cudaStream_t s) {
  mul_kernel<<<blocks_for(n), 256, 0, s>>>(a, b, n, y);
  MLB_CUDA(cudaGetLastError());
}
void op_add(const float* a, const float* b, int n, float* y, cudaStream_t s) {
  add_kernel<<<blocks_for(n), 256, 0, s>>>(a, b, n, y);
  MLB_CUDA(cudaGetLastError());
}
void op_softmax(const float* x, int n, float* y, cudaStream_t s) {
  softmax_kernel<<<1, 1024, 0, s>>>(x, n, y);
  MLB_CUDA(cudaGetLastError());
}
void op_embedding(const float* table, int vocab, int dim, const int* token_dev, int token_host,
                  float* y, cudaStream_t s, bool pdl) {
  launch_pdl(embedding_kernel, dim3(std::max(1u, std::min(blocks_for(dim), 64u))), dim3(256), 0,
             s, pdl, table, vocab, dim, token_dev, token_host, y);
}
void op_rope(float* q, float* k, int nh, int nkv, int D, int neox, const float2* cs_dev,
             cudaStream_t s) {
  rope_kernel<<<blocks_for((long long)(nh + nkv) * (D / 2)), 256, 0, s>>>(q, k, nh, nkv, D, neox,
                                                                          cs_dev);
  MLB_CUDA(cudaGetLastError());
}
void op_kv_write(float* keys, float* values, size_t slot, int n, const float* k, const float* v,
                 cudaStream_t s) {
  kv_write_kernel<<<blocks_for(n), 256, 0, s>>>(keys, values, slot, n, k, v);
  MLB_CUDA(cudaGetLastError());
}
void op_argmax(const float* x, int n, int* out_dev, int* out_dev2, cudaStream_t s, bool pdl) {
  launch_pdl(argmax_kernel, dim3(1), dim3(1024), 0, s, pdl, x, n, out_dev, out_dev2);
}

// (cos, sin) of pos * theta^(-2j/D) for j < D/2, evaluated on the host with the
// reference's float expressions (src/ops.cc:148-151 and 168-170).
void rope_table_host(float theta, int D, int pos0, int npos, float2* out) {
  for (int p = 0; p < npos; ++p) {
    int pos = pos0 + p;
    for (int j = 0; j < D / 2; ++j) {
      float freq = 1.0f / std::pow(theta, static_cast<float>(2 * j) / static_cast<float>(D));
      float ang = static_cast<float>(pos) * freq;
      out[(size_t)p * (D / 2) + j] = make_float2(std::cos(ang), std::sin(ang));
    }
  }
}

float attn_scale(int head_dim) {
  return static_cast<float>(1.0 / static_cast<double>(std::sqrt(static_cast<float>(head_dim))));
}

// ------------------------------------------------------- seeded generator

__global__ void synth_blocks_kernel(int qtype, uint64_t key, float scale, int raw, long long row0,
                                    long long rows, long long blk0, long long nblk,
                                    long long full_cols, const int* src_rows, uint8_t* dst,
                                    size_t pitch) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * nblk) return;
  long long r = i / nblk, b = i - r * nblk;
  long long gr = src_rows ? (long long)src_rows[r] : row0 + r;
  const int bsz = synth::block_bytes(qtype);
  uint8_t* out = dst + (size_t)r * pitch + (size_t)b * bsz;
  uint8_t tmp[34];
  if (gr < 0) {
    for (int j = 0; j < bsz; ++j) tmp[j] = 0;
  } else if (raw) {
    long long nb_full = (full_cols + 31) / 32;
    synth::raw_block(qtype, key, (uint64_t)(gr * nb_full + blk0 + b), tmp);
  } else {
    synth::synth_block(qtype, key, scale, gr, blk0 + b, full_cols, tmp);
  }
  for (int j = 0; j < bsz; ++j) out[j] = tmp[j];
}

void synth_gguf_blocks_rows(int qtype, uint64_t key, float scale, int raw, long long row0,
                            long long rows, long long blk0, long long nblk, long long full_cols,
                            const int* src_rows, uint8_t* dst, size_t dst_pitch,
                            cudaStream_t stream) {
  long long total = rows * nblk;
  if (total <= 0) return;
  synth_blocks_kernel<<<blocks_for(total, 128), 128, 0, stream>>>(
      qtype, key, scale, raw, row0, rows, blk0, nblk, full_cols, src_rows, dst, dst_pitch);
  MLB_CUDA(cudaGetLastError());
}

void synth_gguf_blocks(int qtype, uint64_t key, float scale, int raw, long long row0,
                       long long rows, long long blk0, long long nblk, long long full_cols,
                       uint8_t* dst, size_t dst_pitch, cudaStream_t stream) {
  synth_gguf_blocks_rows(qtype, key, scale, raw, row0, rows, blk0, nblk, full_cols, nullptr, dst,
                         dst_pitch, stream);
}

__global__ void synth_f32_kernel(uint64_t key, float scale, long long row0, long long rows,
                                 long long col0, long long cols, long long full_cols,
                                 float* dst) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  long long r = i / cols, c = i - r * cols;
  dst[i] = synth::fmul(synth::gauss(key, (uint64_t)((row0 + r) * full_cols + col0 + c)), scale);
}

void synth_f32(uint64_t key, float scale, long long row0, long long rows, long long col0,
               long long cols, long long full_cols, float* dst, cudaStream_t stream) {
  long long total = rows * cols;
  if (total <= 0) return;
  synth_f32_kernel<<<blocks_for(total), 256, 0, stream>>>(key, scale, row0, rows, col0, cols,
                                                         full_cols, dst);
  MLB_CUDA(cudaGetLastError());
}

__global__ void fill_kernel(float* p, long long n, float v) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}
void op_fill(float* p, long long n, float v, cudaStream_t s) {
  if (n <= 0) return;
  fill_kernel<<<blocks_for(n), 256, 0, s>>>(p, n, v);
  MLB_CUDA(cudaGetLastError());
}

void qmatrix_synthesize(const QMatrix& m, uint64_t key, float scale, int raw, long long row0,
                        long long full_rows, long long col0, long long full_cols,
                        const int* row_map, cudaStream_t stream) {
  (void)full_rows;
  if (col0 % 32 != 0) invalid("synthesize: column shard must start on a block boundary");
  const size_t pitch = gguf_row_bytes(m.qtype, m.k);
  uint8_t* staging = nullptr;
  const long long nblk = (m.k + 31) / 32;
  MLB_CUDA(cudaMallocAsync(&staging, pitch * (size_t)m.n, stream));
  if (m.qtype == MLB_F32) {
    invalid("synthesize: F32 matrices are generated with synth_f32");
  }
  synth_gguf_blocks_rows(m.qtype, key, scale, raw, row0, m.n, col0 / 32, nblk, full_cols, row_map,
                         staging, pitch, stream);
  qmatrix_repack(m, staging, pitch, nullptr, 0, stream);
  MLB_CUDA(cudaFreeAsync(staging, stream));
}

}  // namespace mlb

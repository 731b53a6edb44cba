// runtime.cu — model weights, decode context and the decode step.
//
// Replaces the device branch of ForwardToken (src/forward.cc:776-794) with
// ForwardLayerDevice (src/forward.cc:711-758), UploadModelWeightsToCuda
// (src/model.cc:345-374) and the CUDA KV cache (src/cuda_kv_cache.cc).
// Where the reference allocates a CudaTensor per op output, looks weights up by
// name string per call and synchronises after every attention kernel, this
// runtime allocates everything once per context, resolves weights to
// pointers once, and records one decode step (5 fused kernels per layer) into
// a CUDA graph whose kernels are chained with programmatic dependent launch.
// Per layer (tensor-parallel size 1):
//   1. QKV GEMV   RMSNorm(x) prologue; +bias, RoPE, q -> q buffer, k/v -> cache
//   2. attention  split-K flash-decode over positions [0, pos]
//   3. wo GEMV    epilogue x' = x + wo . attn
//   4. gate/up    RMSNorm(x') prologue; epilogue h = silu(gate) * up
//   5. down GEMV  epilogue x'' = x' + down . h
// With tensor parallelism, wo and down write partial sums that an NCCL
// all-reduce combines before the residual add, and the vocabulary-sharded
// lm_head logits are all-gathered.
#include <cuda_bf16.h>
#include "runtime.cuh"
#include "sample.cuh"

#include <algorithm>
#include <cstring>
#include <string>

#include "ops.cuh"
#include "synth.h"

namespace mlb {

void DevBuf::alloc(size_t n) {
  reset();
  if (n == 0) return;
  cudaError_t e = cudaMalloc(&p, n);
  if (e != cudaSuccess) {
    p = nullptr;
    (void)cudaGetLastError();
    fail(MLB_ERR_CUDA, "cudaMalloc of " + std::to_string(n) + " bytes failed: " +
                           cudaGetErrorString(e));
  }
  bytes = n;
}
void DevBuf::reset() {
  if (p) cudaFree(p);
  p = nullptr;
  bytes = 0;
}

static void check_nccl(ncclResult_t r, const char* what) {
  if (r != ncclSuccess)
    fail(MLB_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}
#define MLB_NCCL(call) check_nccl((call), #call)

static int round_up(int v, int m) { return (v + m - 1) / m * m; }

// ----------------------------------------------------------- row scatter

__global__ void scatter_rows_kernel(uint8_t* dst, size_t dst_pitch, const uint8_t* src,
                                    size_t src_pitch, size_t row_bytes, const int* dmap,
                                    int nrows) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long total = (long long)nrows * (long long)row_bytes;
  if (i >= total) return;
  int r = (int)(i / (long long)row_bytes);
  size_t c = (size_t)(i - (long long)r * (long long)row_bytes);
  dst[(size_t)dmap[r] * dst_pitch + c] = src[(size_t)r * src_pitch + c];
}

static void scatter_rows(uint8_t* dst, size_t dst_pitch, const RawTensor& src,
                         const std::vector<int>& dmap, cudaStream_t s) {
  if (src.rows == 0) return;
  DevBuf map(dmap.size() * sizeof(int));
  MLB_CUDA(cudaMemcpyAsync(map.p, dmap.data(), dmap.size() * sizeof(int), cudaMemcpyHostToDevice, s));
  long long total = (long long)src.rows * (long long)src.pitch;
  scatter_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      dst, dst_pitch, src.buf.as<uint8_t>(), src.pitch, src.pitch, map.as<int>(), src.rows);
  MLB_CUDA(cudaGetLastError());
  MLB_CUDA(cudaStreamSynchronize(s));
}

// ------------------------------------------------------------------ model

static const char* kKindNames[] = {"token_embedding", "final_norm", "lm_head",
                                   "attention_norm", "wq", "wk", "wv", "bq", "bk", "bv",
                                   "wo", "ffn_norm", "w_gate", "w_up", "w_down"};

static std::string weight_name(int kind, int layer) {
  if (kind < 3) return kKindNames[kind];
  return "layers." + std::to_string(layer) + "." + kKindNames[kind];
}

struct Expect {
  int rows, cols;
  bool f32_only;
};

static Expect expected_shape(const ModelImpl& m, int kind) {
  const mlb_config& c = m.cfg;
  const int qd = c.n_heads * c.head_dim, kvd = c.n_kv_heads * c.head_dim;
  switch (kind) {
    case MLB_W_TOKEN_EMBEDDING: return {c.vocab_size, c.dim, true};
    case MLB_W_FINAL_NORM: case MLB_W_ATTENTION_NORM: case MLB_W_FFN_NORM: return {1, c.dim, true};
    case MLB_W_LM_HEAD: return {c.vocab_size, c.dim, false};
    case MLB_W_WQ: return {qd, c.dim, false};
    case MLB_W_WK: case MLB_W_WV: return {kvd, c.dim, false};
    case MLB_W_BQ: return {1, qd, true};
    case MLB_W_BK: case MLB_W_BV: return {1, kvd, true};
    case MLB_W_WO: return {c.dim, qd, false};
    case MLB_W_GATE: case MLB_W_UP: return {c.hidden_dim, c.dim, false};
    case MLB_W_DOWN: return {c.dim, c.hidden_dim, false};
  }
  out_of_range("weight kind out of range");
}

// Rows of the full tensor this rank keeps ([row0, row0 + rows)); column-sharded
// tensors keep all rows and are cut at repack time.
static void shard_rows(const ModelImpl& m, int kind, int full_rows, int* row0, int* rows) {
  const int D = m.cfg.head_dim;
  switch (kind) {
    case MLB_W_WQ: case MLB_W_BQ:
      *row0 = m.q_head0 * D; *rows = m.q_heads * D; break;
    case MLB_W_WK: case MLB_W_WV: case MLB_W_BK: case MLB_W_BV:
      *row0 = m.kv_head0 * D; *rows = m.kv_heads * D; break;
    case MLB_W_GATE: case MLB_W_UP:
      *row0 = m.ffn_row0; *rows = m.ffn_rows; break;
    case MLB_W_LM_HEAD:
      *row0 = m.vocab_row0; *rows = m.vocab_rows; break;
    default:
      *row0 = 0; *rows = full_rows; break;
  }
  if (kind == MLB_W_BQ || kind == MLB_W_BK || kind == MLB_W_BV) {
    // 1-D tensors: the shard is a column range of the single row
  }
}

mlb_tp_shard tp_plan(const mlb_config& c, int rank, int size) {
  if (size < 1 || rank < 0 || rank >= size) invalid("mlb_model_create: bad tensor-parallel rank/size");
  if (size > 1) {
    if (c.n_heads % size || c.n_kv_heads % size)
      invalid("tensor parallel: n_heads and n_kv_heads must be divisible by the TP size");
    if ((c.n_heads / size * c.head_dim) % 32)
      invalid("tensor parallel: per-rank attention width must be a multiple of 32");
    if (c.hidden_dim % 32 || c.vocab_size % size)
      invalid("tensor parallel: hidden_dim must be a multiple of 32 and vocab divisible by TP size");
  }
  mlb_tp_shard sh{};
  sh.q_heads = c.n_heads / size;
  sh.q_head0 = rank * sh.q_heads;
  sh.kv_heads = c.n_kv_heads / size;
  sh.kv_head0 = rank * sh.kv_heads;
  if (size == 1) {
    sh.ffn_row0 = 0;
    sh.ffn_rows = c.hidden_dim;
  } else {
    const int nb = c.hidden_dim / 32;
    const int b0 = (int)((long long)nb * rank / size), b1 = (int)((long long)nb * (rank + 1) / size);
    sh.ffn_row0 = b0 * 32;
    sh.ffn_rows = (b1 - b0) * 32;
  }
  sh.vocab_rows = c.vocab_size / size;
  sh.vocab_row0 = rank * sh.vocab_rows;
  return sh;
}

ModelImpl* model_create(const mlb_config* cfg, int device, int rank, int size,
                        const void* nccl_id) {
  if (!cfg) invalid("mlb_model_create: null config");
  const mlb_config& c = *cfg;
  if (c.vocab_size <= 0 || c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 ||
      c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 || c.max_seq_len <= 0)
    invalid("mlb_model_create: config dimensions must be positive");
  if (c.n_heads % c.n_kv_heads != 0) invalid("mlb_model_create: n_heads must be divisible by n_kv_heads");
  if (c.head_dim % 4 != 0) invalid("mlb_model_create: head_dim must be a multiple of 4");
  if (!(c.rope_theta > 0.0f) || !std::isfinite(c.rope_theta))
    invalid("Rope: theta must be finite and positive");
  const mlb_tp_shard sh = tp_plan(c, rank, size);
  attn_check_tiled(c.n_heads / size, c.n_kv_heads / size, c.head_dim);
  set_device(device);
  auto m = std::make_unique<ModelImpl>();
  m->cfg = c;
  m->device = device;
  m->tp_rank = rank;
  m->tp_size = size;
  m->neox = c.rope_type == MLB_ROPE_NEOX;
  m->q_heads = sh.q_heads;
  m->q_head0 = sh.q_head0;
  m->kv_heads = sh.kv_heads;
  m->kv_head0 = sh.kv_head0;
  m->ffn_row0 = sh.ffn_row0;
  m->ffn_rows = sh.ffn_rows;
  m->vocab_rows = sh.vocab_rows;
  m->vocab_row0 = sh.vocab_row0;
  m->vocab_pad = m->vocab_rows;
  m->layers.resize(c.n_layers);
  MLB_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  // RoPE table with the reference's float expressions
  std::vector<float2> tab((size_t)c.max_seq_len * (c.head_dim / 2));
  rope_table_host(c.rope_theta, c.head_dim, 0, c.max_seq_len, tab.data());
  m->rope.alloc(tab.size() * sizeof(float2));
  copy_to_device_now(m->rope.p, tab.data(), tab.size() * sizeof(float2));
  if (size > 1) {
    if (!nccl_id) invalid("mlb_model_create: tensor parallelism needs an NCCL id");
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    MLB_NCCL(ncclCommInitRank(&m->comm, size, id, rank));
  }
  return m.release();
}

void model_destroy(ModelImpl* m) {
  if (!m) return;
  if (m->comm) ncclCommDestroy(m->comm);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

static void put_pending(ModelImpl& m, int kind, int layer, RawTensor&& t) {
  m.pending[{kind, kind < 3 ? -1 : layer}] = std::move(t);
}

void model_set_weight(ModelImpl& m, int kind, int layer, int qtype, int rows, int cols,
                      const void* data, size_t bytes) {
  if (m.finalized) invalid("mlb_model_set_weight: model already finalized");
  if (kind < 0 || kind > MLB_W_DOWN) out_of_range("mlb_model_set_weight: kind out of range");
  if (kind >= 3 && (layer < 0 || layer >= m.cfg.n_layers))
    out_of_range("mlb_model_set_weight: layer out of range");
  if (!data) invalid("mlb_model_set_weight: null data for " + weight_name(kind, layer));
  Expect e = expected_shape(m, kind);
  if (rows * cols != e.rows * e.cols || (e.rows > 1 && (rows != e.rows || cols != e.cols)))
    invalid("CUDA forward uploaded weight shape mismatch: " + weight_name(kind, layer));
  if (e.f32_only && qtype != MLB_F32)
    invalid("mlb_model_set_weight: " + weight_name(kind, layer) + " must be F32");
  if (qtype != MLB_F32 && qtype != MLB_Q8_0 && qtype != MLB_Q4_0 && qtype != MLB_Q4_1)
    invalid("CUDA forward Linear unsupported weight type: " + weight_name(kind, layer));
  rows = e.rows;
  cols = e.cols;
  size_t pitch = gguf_row_bytes(qtype, cols);
  if (bytes != pitch * (size_t)rows)
    invalid("mlb_model_set_weight: block count mismatch for " + weight_name(kind, layer));
  set_device(m.device);
  RawTensor t;
  t.qtype = qtype;
  int r0, nr;
  if (rows == 1 && (kind == MLB_W_BQ || kind == MLB_W_BK || kind == MLB_W_BV)) {
    int c0, nc;
    shard_rows(m, kind == MLB_W_BQ ? MLB_W_WQ : MLB_W_WK, cols, &c0, &nc);
    t.rows = 1;
    t.cols = nc;
    t.pitch = (size_t)nc * 4;
    t.buf.alloc(t.pitch);
    copy_to_device_now(t.buf.p, static_cast<const float*>(data) + c0, t.pitch);
  } else {
    shard_rows(m, kind, rows, &r0, &nr);
    t.rows = nr;
    t.cols = cols;
    t.pitch = pitch;
    t.buf.alloc(pitch * (size_t)nr);
    copy_to_device_now(t.buf.p, static_cast<const uint8_t*>(data) + pitch * (size_t)r0,
                        pitch * (size_t)nr);
  }
  put_pending(m, kind, layer, std::move(t));
}

WeightSlot model_weight_slot(const ModelImpl& m, int kind, int layer) {
  if (kind < 0 || kind > MLB_W_DOWN) out_of_range("weight kind out of range");
  if (kind >= 3 && (layer < 0 || layer >= m.cfg.n_layers)) out_of_range("weight layer out of range");
  const Expect e = expected_shape(m, kind);
  WeightSlot w;
  w.rows = e.rows;
  w.cols = e.cols;
  w.f32_only = e.f32_only;
  w.by_cols = kind == MLB_W_BQ || kind == MLB_W_BK || kind == MLB_W_BV;
  if (w.by_cols)
    shard_rows(m, kind == MLB_W_BQ ? MLB_W_WQ : MLB_W_WK, e.cols, &w.first, &w.count);
  else
    shard_rows(m, kind, e.rows, &w.first, &w.count);
  w.name = weight_name(kind, layer);
  return w;
}

void model_put_raw(ModelImpl& m, int kind, int layer, RawTensor&& t) {
  if (m.finalized) invalid("mlb_model_set_weight: model already finalized");
  put_pending(m, kind, layer, std::move(t));
}

static uint64_t stream_id(int kind, int layer) {
  return (uint64_t)kind * (1ull << 20) + (uint64_t)(layer < 0 ? 0 : layer);
}

// Generates the rank's shard of one tensor on the device (see synth.h).
static void synth_tensor(ModelImpl& m, int kind, int layer, int qtype, uint64_t seed) {
  Expect e = expected_shape(m, kind);
  RawTensor t;
  const uint64_t key = synth::stream_key(seed, stream_id(kind, layer));
  cudaStream_t s = m.stream;
  if (kind == MLB_W_FINAL_NORM || kind == MLB_W_ATTENTION_NORM || kind == MLB_W_FFN_NORM) {
    t.qtype = MLB_F32; t.rows = 1; t.cols = e.cols; t.pitch = (size_t)e.cols * 4;
    t.buf.alloc(t.pitch);
    op_fill(t.buf.as<float>(), e.cols, 1.0f, s);
  } else if (kind == MLB_W_TOKEN_EMBEDDING) {
    t.qtype = MLB_F32; t.rows = e.rows; t.cols = e.cols; t.pitch = (size_t)e.cols * 4;
    t.buf.alloc(t.pitch * (size_t)e.rows);
    synth_f32(key, 0.02f, 0, e.rows, 0, e.cols, e.cols, t.buf.as<float>(), s);
  } else if (kind == MLB_W_BQ || kind == MLB_W_BK || kind == MLB_W_BV) {
    int c0, nc;
    shard_rows(m, kind == MLB_W_BQ ? MLB_W_WQ : MLB_W_WK, e.cols, &c0, &nc);
    t.qtype = MLB_F32; t.rows = 1; t.cols = nc; t.pitch = (size_t)nc * 4;
    t.buf.alloc(t.pitch);
    synth_f32(key, 0.02f, 0, 1, c0, nc, e.cols, t.buf.as<float>(), s);
  } else {
    int r0, nr;
    shard_rows(m, kind, e.rows, &r0, &nr);
    t.qtype = qtype; t.rows = nr; t.cols = e.cols; t.pitch = gguf_row_bytes(qtype, e.cols);
    t.buf.alloc(t.pitch * (size_t)nr);
    synth_gguf_blocks(qtype, key, 0.02f, 0, r0, nr, 0, (e.cols + 31) / 32, e.cols,
                      t.buf.as<uint8_t>(), t.pitch, s);
  }
  MLB_CUDA(cudaStreamSynchronize(s));
  put_pending(m, kind, layer, std::move(t));
}

static RawTensor take(ModelImpl& m, int kind, int layer, bool required = true) {
  auto it = m.pending.find({kind, kind < 3 ? -1 : layer});
  if (it == m.pending.end()) {
    if (required) invalid("CUDA forward missing uploaded weight: " + weight_name(kind, layer));
    return RawTensor{};
  }
  RawTensor t = std::move(it->second);
  m.pending.erase(it);
  return t;
}

static void alloc_qmatrix(QMatrix& q, DevBuf& buf, int qtype, int n, int k) {
  qmatrix_geometry(q, qtype, n, k, 1);
  buf.alloc(q.bytes);
  q.data = buf.as<uint8_t>();
}

// Stored row of a logical row inside a head for pair-interleaved NeoX storage.
static int neox_store_row(int l, int D) {
  int head = l / D, i = l % D;
  return head * D + (i < D / 2 ? 2 * i : 2 * (i - D / 2) + 1);
}

static void finalize_layer(ModelImpl& m, int l) {
  LayerPlan& L = m.layers[l];
  const int D = m.cfg.head_dim, dim = m.cfg.dim;
  cudaStream_t s = m.stream;
  RawTensor an = take(m, MLB_W_ATTENTION_NORM, l), fn = take(m, MLB_W_FFN_NORM, l);
  L.attn_norm = std::move(an.buf);
  L.ffn_norm = std::move(fn.buf);
  RawTensor wq = take(m, MLB_W_WQ, l), wk = take(m, MLB_W_WK, l), wv = take(m, MLB_W_WV, l);
  if (wq.qtype != wk.qtype || wq.qtype != wv.qtype)
    invalid("layer " + std::to_string(l) + ": wq, wk and wv must share one quant type");
  // fused QKV: [q | pad | k | pad | v | pad], q/k pair-interleaved for NeoX
  const int qr = m.q_heads * D, kr = m.kv_heads * D;
  L.qkv_k_off = round_up(qr, kTileRows);
  L.qkv_v_off = L.qkv_k_off + round_up(kr, kTileRows);
  const int nq = L.qkv_v_off + round_up(kr, kTileRows);
  {
    const size_t pitch = gguf_row_bytes(wq.qtype, dim);
    DevBuf staging(pitch * (size_t)nq);
    MLB_CUDA(cudaMemsetAsync(staging.p, 0, staging.bytes, s));
    std::vector<int> mq(qr), mk(kr), mv(kr);
    for (int i = 0; i < qr; ++i) mq[i] = m.neox ? neox_store_row(i, D) : i;
    for (int i = 0; i < kr; ++i) {
      mk[i] = L.qkv_k_off + (m.neox ? neox_store_row(i, D) : i);
      mv[i] = L.qkv_v_off + i;
    }
    scatter_rows(staging.as<uint8_t>(), pitch, wq, mq, s);
    scatter_rows(staging.as<uint8_t>(), pitch, wk, mk, s);
    scatter_rows(staging.as<uint8_t>(), pitch, wv, mv, s);
    alloc_qmatrix(L.qkv, L.qkv_buf, wq.qtype, nq, dim);
    qmatrix_repack(L.qkv, staging.as<uint8_t>(), pitch, nullptr, 0, s);
    MLB_CUDA(cudaStreamSynchronize(s));
  }
  RawTensor bq = take(m, MLB_W_BQ, l, false), bk = take(m, MLB_W_BK, l, false),
            bv = take(m, MLB_W_BV, l, false);
  const int nb = (bq.rows > 0) + (bk.rows > 0) + (bv.rows > 0);
  if (nb != 0 && nb != 3) invalid("layer " + std::to_string(l) + ": bq, bk and bv come together");
  if (nb == 3) {
    L.bias.alloc((size_t)(qr + 2 * kr) * 4);
    MLB_CUDA(cudaMemcpyAsync(L.bias.as<float>(), bq.buf.p, (size_t)qr * 4, cudaMemcpyDeviceToDevice, s));
    MLB_CUDA(cudaMemcpyAsync(L.bias.as<float>() + qr, bk.buf.p, (size_t)kr * 4, cudaMemcpyDeviceToDevice, s));
    MLB_CUDA(cudaMemcpyAsync(L.bias.as<float>() + qr + kr, bv.buf.p, (size_t)kr * 4, cudaMemcpyDeviceToDevice, s));
  }
  // wo: this rank's columns (its q heads)
  RawTensor wo = take(m, MLB_W_WO, l);
  alloc_qmatrix(L.wo, L.wo_buf, wo.qtype, dim, qr);
  qmatrix_repack(L.wo, wo.buf.as<uint8_t>(), wo.pitch, nullptr, m.q_head0 * D / 32, s);
  // gate/up interleaved by 8 rows per 16-row tile
  RawTensor wg = take(m, MLB_W_GATE, l), wu = take(m, MLB_W_UP, l);
  if (wg.qtype != wu.qtype) invalid("layer " + std::to_string(l) + ": w_gate and w_up must share one quant type");
  const int F = m.ffn_rows;
  const int ngu = round_up(F, 8) * 2;
  {
    const size_t pitch = gguf_row_bytes(wg.qtype, dim);
    DevBuf staging(pitch * (size_t)ngu);
    MLB_CUDA(cudaMemsetAsync(staging.p, 0, staging.bytes, s));
    std::vector<int> mg(F), mu(F);
    for (int i = 0; i < F; ++i) {
      mg[i] = 16 * (i / 8) + (i % 8);
      mu[i] = 16 * (i / 8) + 8 + (i % 8);
    }
    scatter_rows(staging.as<uint8_t>(), pitch, wg, mg, s);
    scatter_rows(staging.as<uint8_t>(), pitch, wu, mu, s);
    alloc_qmatrix(L.gateup, L.gateup_buf, wg.qtype, ngu, dim);
    qmatrix_repack(L.gateup, staging.as<uint8_t>(), pitch, nullptr, 0, s);
    MLB_CUDA(cudaStreamSynchronize(s));
  }
  RawTensor wd = take(m, MLB_W_DOWN, l);
  alloc_qmatrix(L.down, L.down_buf, wd.qtype, dim, F);
  qmatrix_repack(L.down, wd.buf.as<uint8_t>(), wd.pitch, nullptr, m.ffn_row0 / 32, s);
  MLB_CUDA(cudaStreamSynchronize(s));
}

static void finalize_globals(ModelImpl& m) {
  cudaStream_t s = m.stream;
  RawTensor emb = take(m, MLB_W_TOKEN_EMBEDDING, -1), fnorm = take(m, MLB_W_FINAL_NORM, -1);
  m.embedding = std::move(emb.buf);
  m.final_norm = std::move(fnorm.buf);
  RawTensor lm = take(m, MLB_W_LM_HEAD, -1);
  alloc_qmatrix(m.lm_head, m.lm_head_buf, lm.qtype, m.vocab_rows, m.cfg.dim);
  qmatrix_repack(m.lm_head, lm.buf.as<uint8_t>(), lm.pitch, nullptr, 0, s);
  MLB_CUDA(cudaStreamSynchronize(s));
}

void model_finalize(ModelImpl& m) {
  if (m.finalized) return;
  set_device(m.device);
  for (int l = 0; l < m.cfg.n_layers; ++l)
    if (!m.layers[l].qkv.data) finalize_layer(m, l);
  if (!m.lm_head.data) finalize_globals(m);
  if (!m.pending.empty()) invalid("mlb_model_finalize: unexpected extra weights");
  m.finalized = true;
}

void model_synthesize(ModelImpl& m, int qtype, uint64_t seed, int with_bias) {
  if (m.finalized) invalid("mlb_model_synthesize: model already finalized");
  if (qtype != MLB_Q8_0 && qtype != MLB_Q4_0 && qtype != MLB_Q4_1)
    invalid("mlb_model_synthesize: quant type must be Q8_0, Q4_0 or Q4_1");
  set_device(m.device);
  for (int l = 0; l < m.cfg.n_layers; ++l) {
    for (int kind = MLB_W_ATTENTION_NORM; kind <= MLB_W_DOWN; ++kind) {
      if (!with_bias && (kind == MLB_W_BQ || kind == MLB_W_BK || kind == MLB_W_BV)) continue;
      synth_tensor(m, kind, l, qtype, seed);
    }
    finalize_layer(m, l);
  }
  synth_tensor(m, MLB_W_TOKEN_EMBEDDING, -1, MLB_F32, seed);
  synth_tensor(m, MLB_W_FINAL_NORM, -1, MLB_F32, seed);
  synth_tensor(m, MLB_W_LM_HEAD, -1, qtype, seed);
  finalize_globals(m);
  m.finalized = true;
}

size_t ModelImpl::resident_bytes() const {
  size_t b = embedding.bytes + final_norm.bytes + lm_head_buf.bytes + rope.bytes;
  for (const auto& L : layers)
    b += L.attn_norm.bytes + L.ffn_norm.bytes + L.bias.bytes + L.qkv_buf.bytes + L.wo_buf.bytes +
         L.gateup_buf.bytes + L.down_buf.bytes;
  return b;
}

// GGUF bytes of every matrix one step streams on this rank, plus the small
// fp32 vectors (norms, bias, one embedding row).
size_t ModelImpl::step_weight_bytes() const {
  const mlb_config& c = cfg;
  const int D = c.head_dim;
  size_t b = lm_head.gguf_bytes + (size_t)c.dim * 4 * 2;
  for (const auto& L : layers) {
    const int qtype = L.qkv.qtype;
    b += (size_t)(q_heads + 2 * kv_heads) * D * gguf_row_bytes(qtype, c.dim);
    b += (size_t)c.dim * gguf_row_bytes(L.wo.qtype, q_heads * D);
    b += (size_t)2 * ffn_rows * gguf_row_bytes(L.gateup.qtype, c.dim);
    b += (size_t)c.dim * gguf_row_bytes(L.down.qtype, ffn_rows);
    b += (size_t)c.dim * 4 * 2 + L.bias.bytes;
  }
  return b;
}

// ---------------------------------------------------------------- context

void ContextImpl::release_graphs() {
  if (exec_greedy && exec_greedy != exec) cudaGraphExecDestroy(exec_greedy);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph_greedy && graph_greedy != graph) cudaGraphDestroy(graph_greedy);
  if (graph) cudaGraphDestroy(graph);
  exec = exec_greedy = nullptr;
  graph = graph_greedy = nullptr;
}

ContextImpl::~ContextImpl() {
  if (m) cudaSetDevice(m->device);
  if (stream) cudaStreamSynchronize(stream);
  for (void* p : tp_opened) cudaIpcCloseMemHandle(p);
  release_graphs();
  if (batch) batch_engine_free(batch);
  if (h_scalars) cudaFreeHost(h_scalars);
  if (h_logits) cudaFreeHost(h_logits);
  if (h_tokens) cudaFreeHost(h_tokens);
  if (stream) cudaStreamDestroy(stream);
}

float* ContextImpl::kv_layer(const DevBuf& b, int l) const {
  const mlb_config& cf = m->cfg;
  const size_t layer_elems = (size_t)cf.max_seq_len * m->kv_heads * cf.head_dim;
  return reinterpret_cast<float*>(b.as<uint8_t>() + (size_t)l * layer_elems * (kv_bf16 ? 2 : 4));
}

ContextImpl* context_create(ModelImpl& m, int mode, int kv_type) {
  if (!m.finalized) invalid("mlb_context_create: model is not finalized");
  if (mode != MLB_ATTN_CPU_COMPAT && mode != MLB_ATTN_STANDARD)
    invalid("mlb_context_create: unknown attention mode");
  if (kv_type != MLB_KV_F32 && kv_type != MLB_KV_BF16)
    invalid("mlb_context_create: unknown KV cache type");
  set_device(m.device);
  auto c = std::make_unique<ContextImpl>();
  c->m = &m;
  c->attention_mode = mode;
  MLB_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  const mlb_config& cf = m.cfg;
  c->kv_bf16 = kv_type == MLB_KV_BF16;
  const size_t kv =
      (size_t)cf.n_layers * cf.max_seq_len * m.kv_heads * cf.head_dim * (c->kv_bf16 ? 2 : 4);
  c->keys.alloc(kv);
  c->values.alloc(kv);
  zero_now(c->keys.p, kv);
  zero_now(c->values.p, kv);
  c->xa.alloc((size_t)cf.dim * 4);
  c->xb.alloc((size_t)cf.dim * 4);
  c->y.alloc((size_t)cf.dim * 4);
  c->q.alloc((size_t)m.q_heads * cf.head_dim * 4);
  c->attn.alloc((size_t)m.q_heads * cf.head_dim * 4);
  c->hidden.alloc((size_t)round_up(m.ffn_rows, 8) * 4);
  c->logits_local.alloc((size_t)m.vocab_pad * 4);
  c->logits.alloc((size_t)cf.vocab_size * 4);
  // GEMV workspace: max over matrices of ntiles * nchunks * 16 partials
  size_t pf = 0, nt = 0;
  auto upd = [&](const QMatrix& q) {
    pf = std::max(pf, (size_t)q.ntiles * std::max(q.nchunks, 1) * 16);
    nt = std::max(nt, (size_t)q.ntiles);
  };
  for (const auto& L : m.layers) {
    upd(L.qkv); upd(L.wo); upd(L.gateup); upd(L.down);
  }
  upd(m.lm_head);
  c->gemv_ws.alloc(pf * 4);
  c->gemv_cnt.alloc(nt * 4);
  zero_now(c->gemv_cnt.p, nt * 4);
  c->status.alloc(sizeof(DeviceStatus));
  zero_now(c->status.p, sizeof(DeviceStatus));
  c->ws.partials = c->gemv_ws.as<float>();
  c->ws.partial_floats = pf;
  c->ws.counters = c->gemv_cnt.as<int>();
  c->ws.counter_count = nt;
  c->ws.status = c->status.as<DeviceStatus>();
  c->attn_splits = attn_splits(m.kv_heads, sm_count(m.device), cf.max_seq_len);
  c->attn_ws.alloc(attn_ws_floats(m.q_heads, m.kv_heads, cf.head_dim, c->attn_splits) * 4);
  c->attn_cnt.alloc((size_t)m.kv_heads * 4);
  zero_now(c->attn_cnt.p, (size_t)m.kv_heads * 4);
  // scalars: [0] token, [1] pos, [2] step, [3] spare, then tokens[max_seq]
  c->scalars.alloc((size_t)(4 + cf.max_seq_len) * 4);
  zero_now(c->scalars.p, c->scalars.bytes);
  c->argmax_key.alloc(sizeof(unsigned long long));
  zero_now(c->argmax_key.p, sizeof(unsigned long long));
  MLB_CUDA(cudaMallocHost(&c->h_scalars, 4 * sizeof(int)));
  MLB_CUDA(cudaMallocHost(&c->h_logits, (size_t)cf.vocab_size * 4));
  MLB_CUDA(cudaMallocHost(&c->h_tokens, (size_t)cf.max_seq_len * 4));
  c->plan_step();
  if (c->kv_bf16 && !c->step.ok)
    invalid("mlb_context_create: a bf16 KV cache needs the decode step kernel, which this model "
            "cannot use: " + c->step.why);
  c->use_step = c->step.ok;
  c->build_graph();
  return c.release();
}

// The phase list of one decode step for the persistent kernel, or the reason
// it cannot run this model (then the per-op graph is used).
void ContextImpl::plan_step() {
  step = StepPlan{};
  const mlb_config& cf = m->cfg;
  const int D = cf.head_dim;
  auto no = [&](const std::string& why) {
    step.ok = false;
    step.why = why;
  };
  const bool tp = m->tp_size > 1;
  if (tp && m->tp_size > kMaxTp) return no("more tensor-parallel ranks than the exchange holds");
  if (tp && cf.dim > 8192) return no("tensor parallel: dim above 8192");
  std::string why;
  if (!step_attn_ok(m->q_heads, m->kv_heads, D, &why)) return no(why);
  const int grid = sm_count(m->device);
  if (grid > 256) return no("more than 256 SMs");
  const int qt = m->lm_head.qtype;
  std::vector<const QMatrix*> mats;
  for (const auto& L : m->layers) {
    mats.push_back(&L.qkv);
    mats.push_back(&L.wo);
    mats.push_back(&L.gateup);
    mats.push_back(&L.down);
  }
  mats.push_back(&m->lm_head);
  int scratch = step_attn_scratch(m->q_heads / m->kv_heads, D);
  for (const QMatrix* q : mats) {
    if (q->qtype != qt) return no("projections of more than one quant type");
    if (!step_gemv_ok(*q, grid, &why)) return no(why);
    scratch = std::max(scratch, step_gemv_scratch(*q));
  }
  // every CTA stores its 1/grid slice of the summed residual while staging,
  // which needs the whole input row (dim) staged as one chunk group
  if (tp && cf.n_layers > 0 && (m->layers[0].qkv.ngroups > 1 || m->layers[0].gateup.ngroups > 1))
    return no("tensor parallel with dim above one chunk group");
  const int stride = sb_bytes(qt);
  constexpr size_t kSmemMax = 227 * 1024;
  int stages = 0;
  const int nph = 5 * cf.n_layers + 1;  // per layer QKV, attention, wo, gate/up, down; lm_head
  for (int s = kRingStages; s >= 1 && !stages; --s)
    if (step_smem_bytes(scratch, stride, s, nph) <= kSmemMax) stages = s;
  if (!stages) return no("weight ring and scratch exceed shared memory");
  const size_t smem = step_smem_bytes(scratch, stride, stages, nph);
  if (step_max_blocks_per_sm(qt, m->q_heads / m->kv_heads, smem) < 1)
    return no("the step kernel does not fit on an SM");

  // phases
  std::vector<StepPhase> ph;
  auto gemv = [&](const QMatrix& q, const float* x, const float* norm_w, const EpiParams& e) {
    StepPhase p{};
    p.kind = kPhaseGemv;
    p.g.w = q.data;
    p.g.sbb = sb_bytes(q.qtype);
    p.g.ntiles = q.ntiles;
    p.g.nchunks = q.nchunks;
    p.g.gc = q.gc;
    p.g.ngroups = q.ngroups;
    p.g.nsb = q.nsb;
    p.g.k = q.k;
    p.g.x = x;
    p.g.norm_w = norm_w;
    p.g.eps = cf.rms_norm_eps;
    p.g.epi = e;
    p.g.tp_ar = -1;
    ph.push_back(p);
  };
  int* d_pos = scalars.as<int>() + 1;
  if (tp) setup_tp_exchange();
  // the residual epilogues of wo and w_down (one GPU) or the exchange sums
  // after them (tensor parallel) leave per-tile sums of squares of x, from
  // which the next RMSNorm reads its statistic
  const int ss_n = (cf.dim + kTileRows - 1) / kTileRows;
  ss_x.alloc((size_t)2 * ss_n * 4);
  float* ss_xa = ss_x.as<float>();
  float* ss_xb = ss_xa + ss_n;
  auto ss_in = [&](StepPhase& p, const float* ss) {
    p.g.ss_in = ss;
    p.g.ss_n = ss ? ss_n : 0;
  };
  const TpXchg* tpd = tp ? tp_desc.as<TpXchg>() : nullptr;
  // Tensor parallel: exchange step 2l is layer l's wo partial sums (slot 0),
  // 2l + 1 its w_down partial sums (slot 1). The producing phase adds every
  // rank's partials to the residual (each CTA its tiles) before its barrier,
  // so the consuming phase reads the next residual like a single GPU.
  for (int l = 0; l < cf.n_layers; ++l) {
    const LayerPlan& L = m->layers[l];
    const float* x_in = l == 0 ? nullptr : xa.as<float>();  // null: embedding row
    EpiParams e{};
    e.kind = kEpiQkv;
    e.q_rows = m->q_heads * D;
    e.kv_rows = m->kv_heads * D;
    e.k_off = L.qkv_k_off;
    e.v_off = L.qkv_v_off;
    e.head_dim = D;
    e.neox = m->neox;
    e.bias = L.bias.p ? L.bias.as<float>() : nullptr;
    e.rope = m->rope.as<float2>();
    e.pos = d_pos;
    e.keys = kv_layer(keys, l);
    e.values = kv_layer(values, l);
    e.kv_bf16 = kv_bf16;
    e.q_out = q.as<float>();
    gemv(L.qkv, x_in, L.attn_norm.as<float>(), e);
    if (l > 0) ss_in(ph.back(), ss_xa);

    StepPhase a{};
    a.kind = kPhaseAttn;
    a.at.q = q.as<float>();
    a.at.keys = kv_layer(keys, l);
    a.at.values = kv_layer(values, l);
    a.at.kv_bf16 = kv_bf16;
    a.at.out = attn.as<float>();
    a.at.H = m->q_heads;
    a.at.KV = m->kv_heads;
    a.at.D = D;
    a.at.scale = attn_scale(D);
    a.at.include_current_v = attention_mode == MLB_ATTN_STANDARD;
    ph.push_back(a);

    EpiParams eo{};
    eo.kind = tp ? kEpiTpPartial : kEpiResidual;
    eo.y = xb.as<float>();
    eo.resid = x_in;  // null: embedding row
    eo.ldy = eo.ldr = cf.dim;
    eo.n_out = cf.dim;
    eo.tp = tpd;
    eo.tp_slot = 0;
    eo.ss_out = ss_xb;
    gemv(L.wo, attn.as<float>(), nullptr, eo);
    if (tp) ph.back().g.tp_ar = 2 * l;

    EpiParams eg{};
    eg.kind = kEpiSwiglu;
    eg.y = hidden.as<float>();
    eg.ldy = m->ffn_rows;
    eg.n_out = m->ffn_rows;
    gemv(L.gateup, xb.as<float>(), L.ffn_norm.as<float>(), eg);
    ss_in(ph.back(), ss_xb);

    EpiParams ed{};
    ed.kind = tp ? kEpiTpPartial : kEpiResidual;
    ed.y = xa.as<float>();
    ed.resid = xb.as<float>();
    ed.ldy = ed.ldr = cf.dim;
    ed.n_out = cf.dim;
    ed.tp = tpd;
    ed.tp_slot = 1;
    ed.ss_out = ss_xa;
    gemv(L.down, hidden.as<float>(), nullptr, ed);
    if (tp) ph.back().g.tp_ar = 2 * l + 1;
  }
  EpiParams el{};
  el.kind = kEpiStore;
  el.y = logits.as<float>();
  el.ldy = m->vocab_rows;
  el.n_out = m->vocab_rows;
  el.argmax_key = argmax_key.as<unsigned long long>();
  el.argmax_base = m->vocab_row0;
  el.tp = tpd;
  gemv(m->lm_head, cf.n_layers == 0 ? nullptr : xa.as<float>(), m->final_norm.as<float>(), el);
  if (cf.n_layers > 0) ss_in(ph.back(), ss_xa);

  if ((int)ph.size() != nph) fail(MLB_ERR_INVALID, "decode step kernel: phase count mismatch");
  step_phases.alloc(ph.size() * sizeof(StepPhase));
  copy_to_device_now(step_phases.p, ph.data(), ph.size() * sizeof(StepPhase));
  const std::vector<StepCta> tab = step_cta_table(ph, grid);
  step_cta.alloc(tab.size() * sizeof(StepCta));
  copy_to_device_now(step_cta.p, tab.data(), tab.size() * sizeof(StepCta));
  step_sync.alloc(2 * sizeof(unsigned int));
  zero_now(step_sync.p, step_sync.bytes);
  const int gq = m->q_heads / m->kv_heads;
  step_attn_ws.alloc((size_t)std::max(grid, m->kv_heads) * gq * (D + 4) * 4);  // one record per item
  step_attn_cnt.alloc((size_t)m->kv_heads * 4);
  zero_now(step_attn_cnt.p, step_attn_cnt.bytes);
  step.ok = true;
  step.qtype = qt;
  step.gq = gq;
  step.grid = grid;
  step.stages = stages;
  step.sb_stride = stride;
  step.scratch_bytes = scratch;
  step.smem = smem;
  step.nphases = (int)ph.size();
  step.phases = step_phases.p;
  step.cta = step_cta.p;
}

void ContextImpl::launch_step(cudaStream_t s) {
  StepArgs a{};
  a.phases = static_cast<const StepPhase*>(step.phases);
  a.cta = static_cast<const StepCta*>(step.cta);
  a.nphases = step.nphases;
  a.sb_stride = step.sb_stride;
  a.stages = step.stages;
  a.scratch_bytes = step.scratch_bytes;
  a.embedding = m->embedding.as<float>();
  a.dim = m->cfg.dim;
  int* d_token = scalars.as<int>();
  a.token = d_token;
  a.pos = d_token + 1;
  a.step = d_token + 2;
  a.tokens = d_token + 4;
  a.argmax_key = argmax_key.as<unsigned long long>();
  a.ws = gemv_ws.as<float>();
  a.counters = gemv_cnt.as<int>();
  a.attn_ws = step_attn_ws.as<float>();
  a.attn_counters = step_attn_cnt.as<int>();
  a.sync = step_sync.as<unsigned int>();
  a.status = status.as<DeviceStatus>();
  if (m->tp_size > 1) {
    a.tp = tp_desc.as<TpXchg>();
    a.tp_gen = tp_gen.as<unsigned int>();
    a.tp_steps = 2 * m->cfg.n_layers;
  }
  a.trace = trace_on ? step_trace.as<unsigned long long>() : nullptr;
  step_launch(step, a, s);
}

const float* ContextImpl::logits_dev() const {
  if (use_step && m->tp_size > 1)
    return reinterpret_cast<const float*>(xchg.as<uint8_t>() + tpx.logits_off);
  return logits.as<float>();
}

// Tensor-parallel step kernel: one exchange buffer per rank, its IPC handle
// gathered over the model's NCCL communicator, every other rank's buffer
// opened here (peer access over NVLink). Collective: every rank creates its
// contexts in the same order.
void ContextImpl::setup_tp_exchange() {
  const int n = m->tp_size, me = m->tp_rank;
  const mlb_config& cf = m->cfg;
  auto al = [](long long v) { return (v + 255) / 256 * 256; };
  TpXchg x{};
  x.n = n;
  x.me = me;
  x.dim = cf.dim;
  x.vocab = cf.vocab_size;
  x.parts_off = 0;
  x.logits_off = al(2LL * n * cf.dim * 8);  // tagged 8-byte words
  x.keys_off = al(x.logits_off + (long long)cf.vocab_size * 4);
  x.kflags_off = al(x.keys_off + (long long)n * 8);
  const long long total = al(x.kflags_off + (long long)n * 4);
  xchg.alloc((size_t)total);
  zero_now(xchg.p, (size_t)total);
  cudaIpcMemHandle_t h;
  MLB_CUDA(cudaIpcGetMemHandle(&h, xchg.p));
  DevBuf hb((size_t)n * sizeof(h));
  copy_to_device_now(hb.as<uint8_t>() + (size_t)me * sizeof(h), &h, sizeof(h));
  MLB_NCCL(ncclAllGather(hb.as<uint8_t>() + (size_t)me * sizeof(h), hb.p, sizeof(h), ncclChar,
                         m->comm, stream));
  MLB_CUDA(cudaStreamSynchronize(stream));
  std::vector<cudaIpcMemHandle_t> all(n);
  MLB_CUDA(cudaMemcpy(all.data(), hb.p, (size_t)n * sizeof(h), cudaMemcpyDeviceToHost));
  for (int r = 0; r < n; ++r) {
    if (r == me) {
      x.peers[r] = xchg.as<uint8_t>();
      continue;
    }
    void* p = nullptr;
    MLB_CUDA(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess));
    tp_opened.push_back(p);
    x.peers[r] = static_cast<uint8_t*>(p);
  }
  tpx = x;
  tp_desc.alloc(sizeof(TpXchg));
  copy_to_device_now(tp_desc.p, &x, sizeof(TpXchg));
  tp_gen.alloc(2 * sizeof(unsigned int));
  zero_now(tp_gen.p, 2 * sizeof(unsigned int));
  // every rank's buffer is zeroed and mapped before any rank's first step
  MLB_NCCL(ncclAllReduce(hb.p, hb.p, 1, ncclChar, ncclMax, m->comm, stream));
  MLB_CUDA(cudaStreamSynchronize(stream));
}

// Ends a step: the greedy token of the fused argmax becomes the next input
// token and tokens[step]; position and step advance; the key is cleared.
__global__ void step_finalize_kernel(unsigned long long* key, int* token, int* tokens, int* step,
                                     int* pos) {
  pdl_wait();
  const int t = argmax_index_of(*key);
  *token = t;
  tokens[*step] = t;
  *step += 1;
  *pos += 1;
  *key = 0ull;
}

void ContextImpl::record_step(cudaStream_t s, bool pdl, bool full_logits) {
  const mlb_config& cf = m->cfg;
  const int D = cf.head_dim;
  int* d_token = scalars.as<int>();
  int* d_pos = d_token + 1;
  int* d_step = d_token + 2;
  int* d_tokens = d_token + 4;
  const float scale = attn_scale(D);
  if (use_step) {
    (void)pdl;
    (void)full_logits;  // single GPU: the logits are always written
    launch_step(s);
    kernels_per_step = 1;
    return;
  }
  kernels_per_step = 0;
  op_embedding(m->embedding.as<float>(), cf.vocab_size, cf.dim, d_token, 0, xa.as<float>(), s, pdl);
  ++kernels_per_step;
  for (int l = 0; l < cf.n_layers; ++l) {
    const LayerPlan& L = m->layers[l];
    EpiParams e{};
    e.kind = kEpiQkv;
    e.q_rows = m->q_heads * D;
    e.kv_rows = m->kv_heads * D;
    e.k_off = L.qkv_k_off;
    e.v_off = L.qkv_v_off;
    e.head_dim = D;
    e.neox = m->neox;
    e.bias = L.bias.p ? L.bias.as<float>() : nullptr;
    e.rope = m->rope.as<float2>();
    e.pos = d_pos;
    e.keys = kv_layer(keys, l);
    e.values = kv_layer(values, l);
    e.q_out = q.as<float>();
    NormSpec norm{L.attn_norm.as<float>(), cf.rms_norm_eps};
    gemv_launch(L.qkv, xa.as<float>(), 1, cf.dim, norm, e, ws, s, pdl);
    kernels_per_step += gemv_kernel_count(L.qkv, 1);

    AttnLaunch al;
    al.q = q.as<float>();
    al.keys = kv_layer(keys, l);
    al.values = kv_layer(values, l);
    al.pos_dev = d_pos;
    al.H = m->q_heads;
    al.KV = m->kv_heads;
    al.D = D;
    al.nsplit = attn_splits;
    al.scale = scale;
    al.include_current_v = attention_mode == MLB_ATTN_STANDARD;
    al.ws = attn_ws.as<float>();
    al.counters = attn_cnt.as<int>();
    al.out = attn.as<float>();
    attn_launch(al, s, pdl);
    ++kernels_per_step;

    EpiParams eo{};
    NormSpec none{};
    if (m->tp_size == 1) {
      eo.kind = kEpiResidual;
      eo.y = xb.as<float>();
      eo.resid = xa.as<float>();
      eo.ldy = eo.ldr = cf.dim;
      eo.n_out = cf.dim;
      gemv_launch(L.wo, attn.as<float>(), 1, L.wo.k, none, eo, ws, s, pdl);
      kernels_per_step += gemv_kernel_count(L.wo, 1);
    } else {
      eo.kind = kEpiStore;
      eo.y = y.as<float>();
      eo.ldy = cf.dim;
      eo.n_out = cf.dim;
      gemv_launch(L.wo, attn.as<float>(), 1, L.wo.k, none, eo, ws, s, pdl);
      kernels_per_step += gemv_kernel_count(L.wo, 1);
      MLB_NCCL(ncclAllReduce(y.p, y.p, cf.dim, ncclFloat, ncclSum, m->comm, s));
      op_add(xa.as<float>(), y.as<float>(), cf.dim, xb.as<float>(), s);
      ++kernels_per_step;
    }

    EpiParams eg{};
    eg.kind = kEpiSwiglu;
    eg.y = hidden.as<float>();
    eg.ldy = m->ffn_rows;
    eg.n_out = m->ffn_rows;
    NormSpec fnorm{L.ffn_norm.as<float>(), cf.rms_norm_eps};
    gemv_launch(L.gateup, xb.as<float>(), 1, cf.dim, fnorm, eg, ws, s, pdl);
    kernels_per_step += gemv_kernel_count(L.gateup, 1);

    EpiParams ed{};
    if (m->tp_size == 1) {
      ed.kind = kEpiResidual;
      ed.y = xa.as<float>();
      ed.resid = xb.as<float>();
      ed.ldy = ed.ldr = cf.dim;
      ed.n_out = cf.dim;
      gemv_launch(L.down, hidden.as<float>(), 1, L.down.k, none, ed, ws, s, pdl);
      kernels_per_step += gemv_kernel_count(L.down, 1);
    } else {
      ed.kind = kEpiStore;
      ed.y = y.as<float>();
      ed.ldy = cf.dim;
      ed.n_out = cf.dim;
      gemv_launch(L.down, hidden.as<float>(), 1, L.down.k, none, ed, ws, s, pdl);
      kernels_per_step += gemv_kernel_count(L.down, 1);
      MLB_NCCL(ncclAllReduce(y.p, y.p, cf.dim, ncclFloat, ncclSum, m->comm, s));
      op_add(xb.as<float>(), y.as<float>(), cf.dim, xa.as<float>(), s);
      ++kernels_per_step;
    }
  }
  EpiParams el{};
  el.kind = kEpiStore;
  el.y = m->tp_size == 1 ? logits.as<float>() : logits_local.as<float>();
  el.ldy = m->vocab_rows;
  el.n_out = m->vocab_rows;
  el.argmax_key = argmax_key.as<unsigned long long>();
  el.argmax_base = m->vocab_row0;
  NormSpec fin{m->final_norm.as<float>(), cf.rms_norm_eps};
  gemv_launch(m->lm_head, xa.as<float>(), 1, cf.dim, fin, el, ws, s, pdl);
  kernels_per_step += gemv_kernel_count(m->lm_head, 1);
  if (m->tp_size > 1) {
    // greedy token across the vocabulary shards: max of the packed keys
    MLB_NCCL(ncclAllReduce(argmax_key.p, argmax_key.p, 1, ncclUint64, ncclMax, m->comm, s));
    if (full_logits)
      MLB_NCCL(ncclAllGather(logits_local.p, logits.p, m->vocab_rows, ncclFloat, m->comm, s));
  }
  launch_pdl(step_finalize_kernel, dim3(1), dim3(1), 0, s, pdl && m->tp_size == 1,
             argmax_key.as<unsigned long long>(), d_token, d_tokens, d_step, d_pos);
  ++kernels_per_step;
}

void ContextImpl::build_graph() {
  set_device(m->device);
  release_graphs();
  direct_launch = false;
  if (use_step) {
    // one kernel per step: a graph only saves its launch call; launch directly
    // when the cooperative launch cannot be captured
    cudaGraph_t g = nullptr;
    MLB_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    bool captured = true;
    try {
      record_step(stream, false, true);
    } catch (...) {
      captured = false;
    }
    cudaError_t e = cudaStreamEndCapture(stream, &g);
    if (!captured || e != cudaSuccess || !g ||
        cudaGraphInstantiate(&exec, g, 0) != cudaSuccess) {
      cudaGetLastError();
      if (g) cudaGraphDestroy(g);
      exec = nullptr;
      direct_launch = true;
      kernels_per_step = 1;
      return;
    }
    graph = g;
    exec_greedy = exec;  // same step either way on one GPU
    return;
  }
  for (int full = 1; full >= 0; --full) {
    MLB_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    try {
      record_step(stream, true, full != 0);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    cudaGraph_t& g = full ? graph : graph_greedy;
    MLB_CUDA(cudaStreamEndCapture(stream, &g));
    MLB_CUDA(cudaGraphInstantiate(full ? &exec : &exec_greedy, g, 0));
  }
}

void ContextImpl::replay(bool greedy) {
  if (direct_launch)
    launch_step(stream);
  else
    MLB_CUDA(cudaGraphLaunch(greedy ? exec_greedy : exec, stream));
}

void ContextImpl::set_use_step(bool on) {
  if (on && !step.ok) invalid("decode step kernel unavailable: " + step.why);
  if (!on && kv_bf16)
    invalid("mlb_context_set_step_kernel: a bf16 KV cache runs on the step kernel only");
  set_device(m->device);
  MLB_CUDA(cudaStreamSynchronize(stream));
  use_step = on;
  if (!on) trace_on = false;
  build_graph();
}

void ContextImpl::set_step_trace(bool on) {
  if (on && !use_step) invalid("mlb_context_step_trace: the context is not on the step kernel");
  set_device(m->device);
  MLB_CUDA(cudaStreamSynchronize(stream));
  if (on && !step_trace.p) step_trace.alloc((size_t)step.nphases * step.grid * 2 * 8);
  if (on) zero_now(step_trace.p, step_trace.bytes);
  trace_on = on;
  build_graph();
}

void ContextImpl::read_step_trace(unsigned long long* stamps, size_t cap, int* nphases,
                                  int* grid) {
  if (!trace_on) invalid("mlb_context_step_trace_read: tracing is off");
  *nphases = step.nphases;
  *grid = step.grid;
  const size_t n = step_trace.bytes / 8;
  if (!stamps || cap < n) return;  // a size query
  set_device(m->device);
  MLB_CUDA(cudaStreamSynchronize(stream));
  MLB_CUDA(cudaMemcpy(stamps, step_trace.p, step_trace.bytes, cudaMemcpyDeviceToHost));
  zero_now(step_trace.p, step_trace.bytes);
  for (size_t i = 0; i < n; ++i)
    if (stamps[i] == 0ull)
      invalid("mlb_context_step_trace_read: no whole traced step since the last read");
}

void ContextImpl::check_status() {
  DeviceStatus st{};
  MLB_CUDA(cudaMemcpy(&st, status.p, sizeof(st), cudaMemcpyDeviceToHost));
  if (st.code != 0) {
    // a failed step may leave arrival counters and the argmax key mid-way
    zero_now(gemv_cnt.p, gemv_cnt.bytes);
    zero_now(attn_cnt.p, attn_cnt.bytes);
    zero_now(argmax_key.p, argmax_key.bytes);
    if (step_sync.p) zero_now(step_sync.p, step_sync.bytes);
    if (step_attn_cnt.p) zero_now(step_attn_cnt.p, step_attn_cnt.bytes);
    zero_now(status.p, sizeof(st));
    fail(st.code, "decode step: a device-side check failed (site " + std::to_string(st.where) + ")");
  }
}

static void validate_step(const ContextImpl& c, int token, int pos) {
  const mlb_config& cf = c.m->cfg;
  if (token < 0 || token >= cf.vocab_size) out_of_range("ForwardToken token id out of range");
  if (pos < 0 || pos >= cf.max_seq_len) out_of_range("ForwardToken position out of range");
}

void context_step_async(ContextImpl& c, int token, int pos) {
  validate_step(c, token, pos);
  set_device(c.m->device);
  c.h_scalars[0] = token;
  c.h_scalars[1] = pos;
  c.h_scalars[2] = 0;
  MLB_CUDA(cudaMemcpyAsync(c.scalars.p, c.h_scalars, 3 * sizeof(int), cudaMemcpyHostToDevice, c.stream));
  c.replay(false);
}

void context_forward_token(ContextImpl& c, int token, int pos, float* logits_host) {
  context_step_async(c, token, pos);
  const size_t nb = (size_t)c.m->cfg.vocab_size * 4;
  MLB_CUDA(cudaMemcpyAsync(c.h_logits, c.logits_dev(), nb, cudaMemcpyDeviceToHost, c.stream));
  MLB_CUDA(cudaStreamSynchronize(c.stream));
  c.check_status();
  std::memcpy(logits_host, c.h_logits, nb);
}

void context_decode_greedy(ContextImpl& c, int token, int pos, int n, int* tokens_host) {
  if (n < 0) invalid("mlb_decode_greedy: negative step count");
  if (n == 0) return;
  validate_step(c, token, pos);
  if (pos + n > c.m->cfg.max_seq_len) out_of_range("ForwardToken position out of range");
  set_device(c.m->device);
  c.h_scalars[0] = token;
  c.h_scalars[1] = pos;
  c.h_scalars[2] = 0;
  MLB_CUDA(cudaMemcpyAsync(c.scalars.p, c.h_scalars, 3 * sizeof(int), cudaMemcpyHostToDevice, c.stream));
  for (int i = 0; i < n; ++i) c.replay(true);
  MLB_CUDA(cudaMemcpyAsync(c.h_tokens, c.scalars.as<int>() + 4, (size_t)n * 4,
                           cudaMemcpyDeviceToHost, c.stream));
  MLB_CUDA(cudaStreamSynchronize(c.stream));
  c.check_status();
  std::memcpy(tokens_host, c.h_tokens, (size_t)n * 4);
}

// The step loop of context_decode_greedy with a device sample after each
// step in place of the greedy id (the full-logits step, then sample_launch
// over this rank's complete logits row, which rewrites the next input token
// and the step's entry of the token record).
void context_decode_sample(ContextImpl& c, MtState* st, int* st_out, DeviceStatus* st_status,
                           float temperature, int top_k, int token, int pos, int n,
                           int* tokens_host) {
  if (n < 0) invalid("mlb_decode_sample: negative step count");
  if (n == 0) return;
  validate_step(c, token, pos);
  if (pos + n > c.m->cfg.max_seq_len) out_of_range("ForwardToken position out of range");
  set_device(c.m->device);
  c.h_scalars[0] = token;
  c.h_scalars[1] = pos;
  c.h_scalars[2] = 0;
  MLB_CUDA(cudaMemcpyAsync(c.scalars.p, c.h_scalars, 3 * sizeof(int), cudaMemcpyHostToDevice, c.stream));
  int* d_token = c.scalars.as<int>();
  for (int i = 0; i < n; ++i) {
    c.replay(false);
    sample_launch(c.logits_dev(), c.m->cfg.vocab_size, temperature, top_k, st, st_out, st_status,
                  d_token, d_token + 4, d_token + 2, c.stream);
  }
  MLB_CUDA(cudaMemcpyAsync(c.h_tokens, c.scalars.as<int>() + 4, (size_t)n * 4,
                           cudaMemcpyDeviceToHost, c.stream));
  MLB_CUDA(cudaStreamSynchronize(c.stream));
  c.check_status();
  std::memcpy(tokens_host, c.h_tokens, (size_t)n * 4);
}

void context_reset(ContextImpl& c) {
  set_device(c.m->device);
  MLB_CUDA(cudaMemsetAsync(c.keys.p, 0, c.keys.bytes, c.stream));
  MLB_CUDA(cudaMemsetAsync(c.values.p, 0, c.values.bytes, c.stream));
  MLB_CUDA(cudaStreamSynchronize(c.stream));
}

}  // namespace mlb

namespace mlb {

// Positions [0, n_pos) of every layer of this rank's K and V cache from the
// seeded generator: element (pos, global KV head, d) of layer l is
// gauss(key, (pos * KV + head) * D + d) * scale, keys of streams 15 * 2^20 + l
// (K) and 16 * 2^20 + l (V) -- a decode state at depth n_pos without running
// n_pos steps (the CPU oracle writes the same values).
template <class T>
__device__ __forceinline__ T kv_value(float v);
template <>
__device__ __forceinline__ float kv_value<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 kv_value<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <class T>
__global__ void fill_kv_kernel(T* keys, T* values, int L, int S, int KVl, int KV, int kv0,
                               int D, int n_pos, uint64_t seed, float scale) {
  const long long per_layer = (long long)n_pos * KVl * D;
  const long long total = per_layer * L;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int l = (int)(i / per_layer);
    const long long r = i - (long long)l * per_layer;
    const int p = (int)(r / ((long long)KVl * D));
    const int rem = (int)(r - (long long)p * KVl * D);
    const int h = rem / D, d = rem - h * D;
    const uint64_t idx = ((uint64_t)p * KV + (uint64_t)(kv0 + h)) * D + d;
    const uint64_t kk = synth::stream_key(seed, 15ull * (1ull << 20) + (uint64_t)l);
    const uint64_t kv = synth::stream_key(seed, 16ull * (1ull << 20) + (uint64_t)l);
    const size_t o = (((size_t)l * S + p) * KVl + h) * D + d;
    keys[o] = kv_value<T>(synth::fmul(synth::gauss(kk, idx), scale));
    values[o] = kv_value<T>(synth::fmul(synth::gauss(kv, idx), scale));
  }
}

void fill_kv_rows(void* keys, void* values, bool bf16, const ModelImpl& m, int n_pos,
                  uint64_t seed, float scale, cudaStream_t s) {
  const mlb_config& cf = m.cfg;
  if (n_pos <= 0) return;
  const int grid = sm_count(m.device) * 8;
  if (bf16)
    fill_kv_kernel<<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(keys),
                                       static_cast<__nv_bfloat16*>(values), cf.n_layers,
                                       cf.max_seq_len, m.kv_heads, cf.n_kv_heads, m.kv_head0,
                                       cf.head_dim, n_pos, seed, scale);
  else
    fill_kv_kernel<<<grid, 256, 0, s>>>(static_cast<float*>(keys), static_cast<float*>(values),
                                       cf.n_layers, cf.max_seq_len, m.kv_heads, cf.n_kv_heads,
                                       m.kv_head0, cf.head_dim, n_pos, seed, scale);
  MLB_CUDA(cudaGetLastError());
}

void context_fill_kv(ContextImpl& c, int n_pos, uint64_t seed, float scale) {
  const mlb_config& cf = c.m->cfg;
  if (n_pos < 0 || n_pos > cf.max_seq_len) out_of_range("mlb_context_fill_kv: n_pos out of range");
  set_device(c.m->device);
  fill_kv_rows(c.keys.p, c.values.p, c.kv_bf16, *c.m, n_pos, seed, scale, c.stream);
  MLB_CUDA(cudaStreamSynchronize(c.stream));
}

}  // namespace mlb

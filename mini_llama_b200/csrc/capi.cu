// capi.cu — the extern "C" boundary declared in include/mlb200.h.
//
// Every entry point validates its arguments like the reference entry point it
// replaces (messages follow the reference's wording where its tests grep
// them), turns exceptions into a status code plus a thread-local message, and
// never falls back to a CPU implementation.
#include <cmath>
#include <cstring>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "attention.cuh"
#include "gemv.cuh"
#include "ops.cuh"
#include "qgemm.cuh"
#include "runtime.cuh"
#include "sample.cuh"
#include "synth.h"

namespace mlb {

static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }

void set_device(int device_id) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    fail(MLB_ERR_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
  }
  if (device_id < 0 || device_id >= n)
    invalid("CUDA device id " + std::to_string(device_id) + " is out of range (" +
            std::to_string(n) + " devices)");
  MLB_CUDA(cudaSetDevice(device_id));
}

void zero_now(void* p, size_t bytes) {
  MLB_CUDA(cudaMemset(p, 0, bytes));
  MLB_CUDA(cudaStreamSynchronize(cudaStreamLegacy));
}

void copy_to_device_now(void* dst, const void* src, size_t bytes) {
  MLB_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
  MLB_CUDA(cudaStreamSynchronize(cudaStreamLegacy));
}

int sm_count(int device_id) {
  static int cache[64] = {};
  if (device_id >= 0 && device_id < 64 && cache[device_id]) return cache[device_id];
  int v = 0;
  MLB_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device_id));
  if (device_id >= 0 && device_id < 64) cache[device_id] = v;
  return v;
}

// Model, context and step functions of runtime.cu.
ModelImpl* model_create(const mlb_config* cfg, int device, int rank, int size, const void* id);
mlb_tp_shard tp_plan(const mlb_config& c, int rank, int size);
void model_destroy(ModelImpl* m);
void model_set_weight(ModelImpl& m, int kind, int layer, int qtype, int rows, int cols,
                      const void* data, size_t bytes);
void model_synthesize(ModelImpl& m, int qtype, uint64_t seed, int with_bias);
void model_finalize(ModelImpl& m);
ContextImpl* context_create(ModelImpl& m, int mode, int kv_type);
void context_step_async(ContextImpl& c, int token, int pos);
void context_forward_token(ContextImpl& c, int token, int pos, float* logits_host);
void context_decode_greedy(ContextImpl& c, int token, int pos, int n, int* tokens_host);
void context_decode_sample(ContextImpl& c, MtState* st, int* st_out, DeviceStatus* st_status,
                           float temperature, int top_k, int token, int pos, int n,
                           int* tokens_host);
void context_reset(ContextImpl& c);
void context_fill_kv(ContextImpl& c, int n_pos, uint64_t seed, float scale);

static size_t expected_blocks(int qtype, int out, int in) {
  if (qtype == MLB_F32) return (size_t)out * (size_t)in;
  return (size_t)out * (size_t)((in + 31) / 32);
}

static const char* linear_caller(int qtype) {
  switch (qtype) {
    case MLB_Q8_0: return "CudaQ80Linear";
    case MLB_Q4_0: return "CudaQ40Linear";
    case MLB_Q4_1: return "CudaQ41Linear";
    default: return "CudaLinear";
  }
}

// Shape checks of ValidateQuantLinearShape, src/cuda_quant.cu:206-223.
static void validate_linear(int qtype, int rows, int in, size_t block_count, int out) {
  const std::string caller = linear_caller(qtype);
  if (qtype != MLB_F32 && qtype != MLB_Q8_0 && qtype != MLB_Q4_0 && qtype != MLB_Q4_1)
    invalid(caller + ": unsupported quant type " + std::to_string(qtype));
  if (rows <= 0 || in <= 0 || out <= 0) invalid(caller + ": empty tensors are not supported");
  size_t exp = expected_blocks(qtype, out, in);
  if (block_count != exp)
    invalid(caller + ": block count mismatch: expected " + std::to_string(exp) + ", got " +
            std::to_string(block_count));
}

static size_t weight_bytes(int qtype, int out, int in) {
  return (size_t)out * gguf_row_bytes(qtype, in);
}

struct QMatrixHandle {
  QMatrix q;
  DevBuf buf;
  int device = 0;
  GemvWorkspace ws;
  DevBuf wsbuf, cnt, status;
  // tensor-core GEMM (batches): staged activations and split-tile scratch,
  // allocated on first use
  TcWorkspace tcws;
  DevBuf tc_staged, tc_parts, tc_cnt;
};

}  // namespace mlb

using namespace mlb;

struct mlb_qmatrix : QMatrixHandle {};
struct mlb_model {
  ModelImpl* impl;
};
struct mlb_context {
  ContextImpl* impl;
};

extern "C" {

const char* mlb_last_error(void) { return g_last_error.c_str(); }

int mlb_built(void) { return 1; }

int mlb_device_count(int* count) {
  return guarded([&] {
    if (!count) invalid("mlb_device_count: null output");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    *count = n;
  });
}

int mlb_linear(int qtype, const float* x_dev, int rows, int in_features, const void* w_dev,
               size_t block_count, int out_features, float* y_dev, int device_id, void* stream) {
  return guarded([&] {
    validate_linear(qtype, rows, in_features, block_count, out_features);
    if (!x_dev || !w_dev || !y_dev)
      invalid(std::string(linear_caller(qtype)) + ": device weight pointer is null");
    set_device(device_id);
    gemv_gguf(qtype, x_dev, rows, in_features, w_dev, out_features, y_dev,
              static_cast<cudaStream_t>(stream));
  });
}

static void linear_host_common(int qtype, const float* x, int rows, int in, const void* w_dev,
                               int out, const float* bias, float* y, cudaStream_t s) {
  DevBuf xd((size_t)rows * in * 4), yd((size_t)rows * out * 4);
  MLB_CUDA(cudaMemcpyAsync(xd.p, x, xd.bytes, cudaMemcpyHostToDevice, s));
  gemv_gguf(qtype, xd.as<float>(), rows, in, w_dev, out, yd.as<float>(), s);
  MLB_CUDA(cudaMemcpyAsync(y, yd.p, yd.bytes, cudaMemcpyDeviceToHost, s));
  MLB_CUDA(cudaStreamSynchronize(s));
  if (bias)  // AddBiasInPlace, src/cuda_quant.cu:135-147
    for (int r = 0; r < rows; ++r)
      for (int j = 0; j < out; ++j) y[(size_t)r * out + j] += bias[j];
}

int mlb_linear_host(int qtype, const float* x, int rows, int in_features, const void* w,
                    size_t block_count, int out_features, const float* bias, float* y,
                    int device_id) {
  return guarded([&] {
    validate_linear(qtype, rows, in_features, block_count, out_features);
    if (!x || !w || !y) invalid(std::string(linear_caller(qtype)) + ": null host pointer");
    set_device(device_id);
    DevBuf wd(weight_bytes(qtype, out_features, in_features));
    copy_to_device_now(wd.p, w, wd.bytes);
    linear_host_common(qtype, x, rows, in_features, wd.p, out_features, bias, y, nullptr);
  });
}

int mlb_linear_device_weight(int qtype, const float* x, int rows, int in_features,
                             const void* w_dev, size_t block_count, int out_features,
                             const float* bias, float* y, int device_id) {
  return guarded([&] {
    validate_linear(qtype, rows, in_features, block_count, out_features);
    if (!w_dev) invalid(std::string(linear_caller(qtype)) + ": device weight pointer is null");
    if (!x || !y) invalid(std::string(linear_caller(qtype)) + ": null host pointer");
    set_device(device_id);
    linear_host_common(qtype, x, rows, in_features, w_dev, out_features, bias, y, nullptr);
  });
}

int mlb_rmsnorm(const float* x, const float* w, int n, float eps, float* y, int device_id,
                void* stream) {
  return guarded([&] {
    if (n <= 0) invalid("RmsNorm: expected 1D tensors");
    if (!x || !w || !y) invalid("RmsNorm: null pointer");
    set_device(device_id);
    op_rmsnorm(x, w, n, eps, y, static_cast<cudaStream_t>(stream));
  });
}

int mlb_silu(const float* x, int n, float* y, int device_id, void* stream) {
  return guarded([&] {
    if (n < 0 || (n > 0 && (!x || !y))) invalid("Silu: bad arguments");
    set_device(device_id);
    if (n) op_silu(x, n, y, static_cast<cudaStream_t>(stream));
  });
}

int mlb_mul(const float* a, const float* b, int n, float* y, int device_id, void* stream) {
  return guarded([&] {
    if (n < 0 || (n > 0 && (!a || !b || !y))) invalid("ElementwiseMul: bad arguments");
    set_device(device_id);
    if (n) op_mul(a, b, n, y, static_cast<cudaStream_t>(stream));
  });
}

int mlb_add(const float* a, const float* b, int n, float* y, int device_id, void* stream) {
  return guarded([&] {
    if (n < 0 || (n > 0 && (!a || !b || !y))) invalid("ElementwiseAdd: bad arguments");
    set_device(device_id);
    if (n) op_add(a, b, n, y, static_cast<cudaStream_t>(stream));
  });
}

int mlb_softmax(const float* x, int n, float* y, int device_id, void* stream) {
  return guarded([&] {
    if (n <= 0) invalid("Softmax: cannot compute Softmax of empty tensor");
    set_device(device_id);
    op_softmax(x, n, y, static_cast<cudaStream_t>(stream));
  });
}

int mlb_embedding(const float* table, int vocab, int dim, int token, float* y, int device_id,
                  void* stream) {
  return guarded([&] {
    if (vocab <= 0 || dim <= 0) invalid("EmbeddingLookup: empty table");
    if (token < 0 || token >= vocab) out_of_range("ForwardToken token id out of range");
    set_device(device_id);
    op_embedding(table, vocab, dim, nullptr, token, y, static_cast<cudaStream_t>(stream), false);
  });
}

int mlb_rope(float* q, float* k, int n_heads, int n_kv_heads, int head_dim, int pos, float theta,
             int rope_type, int device_id, void* stream) {
  return guarded([&] {
    if (pos < 0) out_of_range("Rope: position must be positive");
    if (!(theta > 0.0f) || !std::isfinite(theta)) invalid("Rope: theta must be finite and positive");
    if (head_dim <= 0 || head_dim % 2 != 0)
      invalid("Rope: head_dim must be positive and even, got " + std::to_string(head_dim));
    if (n_heads < 0 || n_kv_heads < 0) invalid("Rope: negative head count");
    set_device(device_id);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    std::vector<float2> tab(head_dim / 2);
    rope_table_host(theta, head_dim, pos, 1, tab.data());
    DevBuf cs(tab.size() * sizeof(float2));
    MLB_CUDA(cudaMemcpyAsync(cs.p, tab.data(), cs.bytes, cudaMemcpyHostToDevice, s));
    op_rope(q, k, n_heads, n_kv_heads, head_dim, rope_type == MLB_ROPE_NEOX, cs.as<float2>(), s);
    MLB_CUDA(cudaStreamSynchronize(s));
  });
}

int mlb_argmax(const float* x, int n, int* index_host, int device_id, void* stream) {
  return guarded([&] {
    if (n <= 0) invalid("ArgMax: cannot compute ArgMax of empty tensor");
    if (!index_host) invalid("ArgMax: null output");
    set_device(device_id);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    DevBuf out(sizeof(int));
    op_argmax(x, n, out.as<int>(), nullptr, s, false);
    MLB_CUDA(cudaMemcpyAsync(index_host, out.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    MLB_CUDA(cudaStreamSynchronize(s));
  });
}

// CudaKvCache::ValidateIndices / WriteDevice checks, src/cuda_kv_cache.cc:137-163, 295-305.
int mlb_kv_write(float* keys, float* values, int n_layers, int max_seq_len, int n_kv_heads,
                 int head_dim, int layer, int pos, const float* k, const float* v, int device_id,
                 void* stream) {
  return guarded([&] {
    if (!keys || !values || n_layers <= 0 || max_seq_len <= 0)
      invalid("CudaKvCache: cache is empty");
    if (layer < 0 || layer >= n_layers) out_of_range("CudaKvCache layer out of range");
    if (pos < 0 || pos >= max_seq_len) out_of_range("CudaKvCache position out of range");
    if (!k || !v || n_kv_heads <= 0 || head_dim <= 0)
      out_of_range("CudaKvCache::WriteDevice tensor shape does not match cache shape");
    set_device(device_id);
    size_t slot = ((size_t)layer * max_seq_len + pos) * (size_t)n_kv_heads * head_dim;
    op_kv_write(keys, values, slot, n_kv_heads * head_dim, k, v, static_cast<cudaStream_t>(stream));
  });
}

// ValidateAttentionDeviceInputs, src/cuda_attention.cu:69-97.
int mlb_attention_decode(const float* q, const float* keys, const float* values, int n_layers,
                         int max_seq_len, int layer, int pos, int n_heads, int n_kv_heads,
                         int head_dim, int mode, float* out, int device_id, void* stream) {
  return guarded([&] {
    if (!keys || !values || n_layers <= 0 || max_seq_len <= 0)
      invalid("CudaAttentionDecodeDeviceInput: CUDA KV cache is empty");
    if (layer < 0 || layer >= n_layers) out_of_range("CudaAttentionDecodeDeviceInput: layer out of range");
    if (pos < 0 || pos >= max_seq_len) out_of_range("CudaAttentionDecodeDeviceInput: position out of range");
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0)
      invalid("CudaAttentionDecodeDeviceInput: head counts and head_dim must be positive");
    if (n_heads % n_kv_heads != 0)
      invalid("CudaAttentionDecodeDeviceInput: n_heads must be divisible by n_kv_heads");
    if (mode != MLB_ATTN_CPU_COMPAT && mode != MLB_ATTN_STANDARD)
      invalid("CudaAttentionDecodeDeviceInput: unknown attention mode");
    if (!q || !out) invalid("CudaAttentionDecodeDeviceInput: null pointer");
    attn_check(n_heads, n_kv_heads, head_dim);
    set_device(device_id);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int nsplit = attn_splits(n_kv_heads, sm_count(device_id), pos + 1);
    DevBuf ws(attn_ws_floats(n_heads, n_kv_heads, head_dim, nsplit) * 4);
    DevBuf cnt((size_t)n_kv_heads * 4);
    MLB_CUDA(cudaMemsetAsync(cnt.p, 0, cnt.bytes, s));
    AttnLaunch l;
    size_t layer_off = (size_t)layer * max_seq_len * n_kv_heads * head_dim;
    l.q = q;
    l.keys = keys + layer_off;
    l.values = values + layer_off;
    l.pos_host = pos;
    l.H = n_heads;
    l.KV = n_kv_heads;
    l.D = head_dim;
    l.nsplit = nsplit;
    l.scale = attn_scale(head_dim);
    l.include_current_v = mode == MLB_ATTN_STANDARD;
    l.ws = ws.as<float>();
    l.counters = cnt.as<int>();
    l.out = out;
    attn_launch(l, s, false);
    MLB_CUDA(cudaStreamSynchronize(s));
  });
}

// ---------------------------------------------------------- prepared weights

static void qmatrix_tc_ws(mlb_qmatrix& h);

static void qmatrix_ws(mlb_qmatrix& h) {
  size_t pf = (size_t)h.q.ntiles * std::max(h.q.nchunks, 1) * 16 * kMaxBatch;
  h.wsbuf.alloc(pf * 4);
  h.cnt.alloc((size_t)h.q.ntiles * 4);
  zero_now(h.cnt.p, h.cnt.bytes);
  h.status.alloc(sizeof(DeviceStatus));
  zero_now(h.status.p, h.status.bytes);
  h.ws.partials = h.wsbuf.as<float>();
  h.ws.partial_floats = pf;
  h.ws.counters = h.cnt.as<int>();
  h.ws.counter_count = h.q.ntiles;
  h.ws.status = h.status.as<DeviceStatus>();
  // the tensor-core GEMM's scratch too, so that no call allocates (calls may
  // be captured in a CUDA graph)
  if (h.q.qtype != MLB_F32) qmatrix_tc_ws(h);
}

int mlb_qmatrix_create(int qtype, const void* w, int w_is_host, int out_features, int in_features,
                       int device_id, mlb_qmatrix** out) {
  return guarded([&] {
    if (!out || !w) invalid("mlb_qmatrix_create: null pointer");
    set_device(device_id);
    auto h = std::make_unique<mlb_qmatrix>();
    h->device = device_id;
    qmatrix_geometry(h->q, qtype, out_features, in_features, kMaxBatch);
    h->buf.alloc(h->q.bytes);
    h->q.data = h->buf.as<uint8_t>();
    const size_t pitch = gguf_row_bytes(qtype, in_features);
    const uint8_t* src = static_cast<const uint8_t*>(w);
    DevBuf tmp;
    if (w_is_host) {
      tmp.alloc(pitch * (size_t)out_features);
      copy_to_device_now(tmp.p, w, tmp.bytes);
      src = tmp.as<uint8_t>();
    }
    qmatrix_repack(h->q, src, pitch, nullptr, 0, nullptr);
    MLB_CUDA(cudaDeviceSynchronize());
    qmatrix_ws(*h);
    *out = h.release();
  });
}

int mlb_qmatrix_synthesize(int qtype, int out_features, int in_features, uint64_t seed,
                           uint64_t stream_id, int raw, int device_id, mlb_qmatrix** out) {
  return guarded([&] {
    if (!out) invalid("mlb_qmatrix_synthesize: null output");
    if (qtype == MLB_F32) invalid("mlb_qmatrix_synthesize: quantised types only");
    set_device(device_id);
    auto h = std::make_unique<mlb_qmatrix>();
    h->device = device_id;
    qmatrix_geometry(h->q, qtype, out_features, in_features, kMaxBatch);
    h->buf.alloc(h->q.bytes);
    h->q.data = h->buf.as<uint8_t>();
    qmatrix_synthesize(h->q, synth::stream_key(seed, stream_id), 0.02f, raw, 0, out_features, 0,
                       in_features, nullptr, nullptr);
    MLB_CUDA(cudaDeviceSynchronize());
    qmatrix_ws(*h);
    *out = h.release();
  });
}

static void qmatrix_tc_gemm(mlb_qmatrix& h, const float* x, int rows, float* y, cudaStream_t s);

int mlb_qmatrix_gemv(mlb_qmatrix* m, const float* x, int rows, float* y, void* stream) {
  return guarded([&] {
    if (!m || !x || !y) invalid("mlb_qmatrix_gemv: null pointer");
    if (rows <= 0) invalid("mlb_qmatrix_gemv: rows must be positive");
    set_device(m->device);
    if (rows > kMaxBatch && m->q.qtype != MLB_F32) {
      // a batch: one pass of the weights through the tensor cores
      qmatrix_tc_gemm(*m, x, rows, y, static_cast<cudaStream_t>(stream));
      return;
    }
    EpiParams e{};
    e.kind = kEpiStore;
    e.y = y;
    e.ldy = m->q.n;
    e.n_out = m->q.n;
    gemv_launch(m->q, x, rows, m->q.k, NormSpec{}, e, m->ws, static_cast<cudaStream_t>(stream),
                false);
  });
}

// Scratch of the tensor-core GEMM for up to kTcMaxMp rows per pass.
static void qmatrix_tc_ws(mlb_qmatrix& h) {
  if (h.tc_staged.p) return;
  const int grid = sm_count(h.device);
  h.tc_staged.alloc((size_t)h.q.nchunks * tc_chunk_bytes(kTcMaxMp));
  const size_t pf = tc_partial_floats(h.q, kTcMaxMp, grid);
  h.tc_parts.alloc(pf * 4);
  const int nc = tc_counter_count(h.q);
  h.tc_cnt.alloc((size_t)nc * 4);
  zero_now(h.tc_cnt.p, h.tc_cnt.bytes);
  h.tcws.partials = h.tc_parts.as<float>();
  h.tcws.partial_floats = pf;
  h.tcws.counters = h.tc_cnt.as<int>();
  h.tcws.counter_count = nc;
  h.tcws.status = h.ws.status;
}

// y = W x through the tensor-core GEMM, kTcMaxMp rows per pass.
static void qmatrix_tc_gemm(mlb_qmatrix& h, const float* x, int rows, float* y, cudaStream_t s) {
  if (h.q.qtype == MLB_F32) invalid("mlb_qmatrix_gemm: quantised types only");
  qmatrix_tc_ws(h);
  for (int r0 = 0; r0 < rows; r0 += kTcMaxMp) {
    const int n = std::min(kTcMaxMp, rows - r0);
    tc_stage_launch(x + (size_t)r0 * h.q.k, h.q.k, n, h.q.k, h.q.nchunks, nullptr, 0.0f, nullptr,
                    h.tc_staged.as<uint8_t>(), s, r0 > 0);
    BEpi e{};
    e.kind = kEpiStore;
    e.y = y + (size_t)r0 * h.q.n;
    e.ldy = h.q.n;
    e.n_out = h.q.n;
    tc_gemm_launch(h.q, h.tc_staged.as<uint8_t>(), n, e, h.tcws, s, 0, true);
  }
}

int mlb_qmatrix_gemm(mlb_qmatrix* m, const float* x, int rows, float* y, void* stream) {
  return guarded([&] {
    if (!m || !x || !y) invalid("mlb_qmatrix_gemm: null pointer");
    if (rows <= 0) invalid("mlb_qmatrix_gemm: rows must be positive");
    set_device(m->device);
    qmatrix_tc_gemm(*m, x, rows, y, static_cast<cudaStream_t>(stream));
  });
}

int mlb_qmatrix_dequant(const mlb_qmatrix* m, float* out_dev, void* stream) {
  return guarded([&] {
    if (!m || !out_dev) invalid("mlb_qmatrix_dequant: null pointer");
    set_device(m->device);
    qmatrix_dequant(m->q, out_dev, static_cast<cudaStream_t>(stream));
  });
}

size_t mlb_qmatrix_bytes(const mlb_qmatrix* m) { return m ? m->q.gguf_bytes : 0; }

int mlb_qmatrix_destroy(mlb_qmatrix* m) {
  return guarded([&] {
    if (m) {
      cudaSetDevice(m->device);
      delete m;
    }
  });
}

// ------------------------------------------------------------- model/context

int mlb_tp_plan(const mlb_config* cfg, int tp_rank, int tp_size, mlb_tp_shard* out) {
  return guarded([&] {
    if (!cfg || !out) invalid("mlb_tp_plan: null pointer");
    *out = tp_plan(*cfg, tp_rank, tp_size);
  });
}

int mlb_model_create(const mlb_config* cfg, int device_id, int tp_rank, int tp_size,
                     const void* nccl_id, mlb_model** out) {
  return guarded([&] {
    if (!out) invalid("mlb_model_create: null output");
    ModelImpl* impl = model_create(cfg, device_id, tp_rank, tp_size, nccl_id);
    *out = new mlb_model{impl};
  });
}

int mlb_model_set_weight(mlb_model* m, int kind, int layer, int qtype, int rows, int cols,
                         const void* host_data, size_t bytes) {
  return guarded([&] {
    if (!m) invalid("mlb_model_set_weight: null model");
    model_set_weight(*m->impl, kind, layer, qtype, rows, cols, host_data, bytes);
  });
}

int mlb_model_synthesize(mlb_model* m, int qtype, uint64_t seed, int with_bias) {
  return guarded([&] {
    if (!m) invalid("mlb_model_synthesize: null model");
    model_synthesize(*m->impl, qtype, seed, with_bias);
  });
}

int mlb_gguf_read_config(const char* path, mlb_config* out) {
  return guarded([&] {
    if (!path || !out) invalid("mlb_gguf_read_config: null argument");
    std::unique_ptr<GgufFile, void (*)(GgufFile*)> g(gguf_open(path), gguf_close);
    *out = gguf_config(*g);
  });
}

int mlb_model_load_gguf(const char* path, int device_id, int tp_rank, int tp_size,
                        const void* nccl_id, int max_seq_len, mlb_model** out,
                        size_t* bytes_uploaded) {
  return guarded([&] {
    if (!path || !out) invalid("mlb_model_load_gguf: null argument");
    if (max_seq_len < 0) invalid("mlb_model_load_gguf: negative max_seq_len");
    std::unique_ptr<GgufFile, void (*)(GgufFile*)> g(gguf_open(path), gguf_close);
    mlb_config cfg = gguf_config(*g);
    if (max_seq_len > 0) cfg.max_seq_len = max_seq_len;
    std::unique_ptr<ModelImpl, void (*)(ModelImpl*)> impl(
        model_create(&cfg, device_id, tp_rank, tp_size, nccl_id), model_destroy);
    const size_t n = gguf_upload(*impl, *g);
    model_finalize(*impl);
    if (bytes_uploaded) *bytes_uploaded = n;
    *out = new mlb_model{impl.release()};
  });
}

int mlb_model_finalize(mlb_model* m) {
  return guarded([&] {
    if (!m) invalid("mlb_model_finalize: null model");
    model_finalize(*m->impl);
  });
}

int mlb_model_destroy(mlb_model* m) {
  return guarded([&] {
    if (m) {
      model_destroy(m->impl);
      delete m;
    }
  });
}

int mlb_model_bytes(const mlb_model* m, size_t* resident, size_t* per_step) {
  return guarded([&] {
    if (!m) invalid("mlb_model_bytes: null model");
    if (resident) *resident = m->impl->resident_bytes();
    if (per_step) *per_step = m->impl->step_weight_bytes();
  });
}

int mlb_context_create(mlb_model* m, int attention_mode, mlb_context** out) {
  return guarded([&] {
    if (!m || !out) invalid("mlb_context_create: null pointer");
    *out = new mlb_context{context_create(*m->impl, attention_mode, MLB_KV_F32)};
  });
}

int mlb_context_create_kv(mlb_model* m, int attention_mode, int kv_type, mlb_context** out) {
  return guarded([&] {
    if (!m || !out) invalid("mlb_context_create: null pointer");
    *out = new mlb_context{context_create(*m->impl, attention_mode, kv_type)};
  });
}

int mlb_context_destroy(mlb_context* c) {
  return guarded([&] {
    if (c) {
      delete c->impl;
      delete c;
    }
  });
}

int mlb_context_reset(mlb_context* c) {
  return guarded([&] {
    if (!c) invalid("mlb_context_reset: null context");
    context_reset(*c->impl);
  });
}

int mlb_context_fill_kv(mlb_context* c, int n_pos, uint64_t seed, float scale) {
  return guarded([&] {
    if (!c) invalid("mlb_context_fill_kv: null context");
    context_fill_kv(*c->impl, n_pos, seed, scale);
  });
}

int mlb_forward_token(mlb_context* c, int token, int pos, float* logits_host) {
  return guarded([&] {
    if (!c || !logits_host) invalid("ForwardToken: null pointer");
    context_forward_token(*c->impl, token, pos, logits_host);
  });
}

int mlb_forward_token_device(mlb_context* c, int token, int pos, const float** logits_dev) {
  return guarded([&] {
    if (!c) invalid("ForwardToken: null context");
    context_step_async(*c->impl, token, pos);
    if (logits_dev) *logits_dev = c->impl->logits_dev();
  });
}

int mlb_context_sync(mlb_context* c) {
  return guarded([&] {
    if (!c) invalid("mlb_context_sync: null context");
    set_device(c->impl->m->device);
    MLB_CUDA(cudaStreamSynchronize(c->impl->stream));
    c->impl->check_status();
  });
}

// ------------------------------------------------------------------ sampling

struct mlb_sampler {
  int device = 0;
  mlb::DevBuf state;   // MtState
  mlb::DevBuf out;     // int: the last sample
  mlb::DevBuf status;  // DeviceStatus: a non-finite logit
  cudaStream_t stream = nullptr;
};

namespace {

// MiniSampler::Sample's parameter checks (src/sampler.cc:28-41, 175-178), on
// the host; the finiteness of the logits is checked on the device.
void validate_sampling(int n, float temperature, int top_k) {
  if (n <= 0) mlb::invalid("sampler: cannot sample from empty logits");
  if (top_k < 0) mlb::invalid("sampler: top_k must be non-negative");
  if (!std::isfinite(temperature) || temperature < 0.0f)
    mlb::invalid("Sampler: temperature must be finite and non-negative");
  const bool greedy = temperature < 1e-6f || top_k == 1;
  if (!greedy && top_k > 1 && std::min(top_k, n) > mlb::kSampleMaxTopK)
    mlb::invalid("sampler: top_k above " + std::to_string(mlb::kSampleMaxTopK) +
                 " is not sampled on the device");
}

void check_sampler_status(mlb_sampler* s) {
  mlb::DeviceStatus st{};
  MLB_CUDA(cudaMemcpy(&st, s->status.p, sizeof(st), cudaMemcpyDeviceToHost));
  if (st.code != 0) {
    zero_now(s->status.p, sizeof(st));
    mlb::invalid("sampler: logits must be finite");
  }
}

}  // namespace

int mlb_sampler_create(int device_id, unsigned int seed, mlb_sampler** out) {
  return guarded([&] {
    if (!out) invalid("mlb_sampler_create: null output");
    *out = nullptr;
    set_device(device_id);
    auto s = std::make_unique<mlb_sampler>();
    s->device = device_id;
    if (seed == 0) seed = std::random_device{}();  // MiniSampler(0): a random seed
    MtState h;
    mt_seed(seed, &h);
    s->state.alloc(sizeof(MtState));
    copy_to_device_now(s->state.p, &h, sizeof(MtState));
    s->out.alloc(sizeof(int));
    s->status.alloc(sizeof(DeviceStatus));
    zero_now(s->status.p, sizeof(DeviceStatus));
    MLB_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    *out = s.release();
  });
}

int mlb_sampler_destroy(mlb_sampler* s) {
  return guarded([&] {
    if (!s) return;
    set_device(s->device);
    if (s->stream) cudaStreamDestroy(s->stream);
    delete s;
  });
}

int mlb_sample(mlb_sampler* s, const float* logits_dev, int n, float temperature, int top_k,
               int* out_id) {
  return guarded([&] {
    if (!s || !out_id || (n > 0 && !logits_dev)) invalid("mlb_sample: null pointer");
    validate_sampling(n, temperature, top_k);
    set_device(s->device);
    sample_launch(logits_dev, n, temperature, top_k, s->state.as<MtState>(), s->out.as<int>(),
                  s->status.as<DeviceStatus>(), nullptr, nullptr, nullptr, s->stream);
    MLB_CUDA(cudaMemcpyAsync(out_id, s->out.p, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
    MLB_CUDA(cudaStreamSynchronize(s->stream));
    check_sampler_status(s);
  });
}

int mlb_decode_sample(mlb_context* c, mlb_sampler* s, float temperature, int top_k, int token,
                      int pos, int n_steps, int* tokens_host) {
  return guarded([&] {
    if (!c || !s || (n_steps > 0 && !tokens_host)) invalid("mlb_decode_sample: null pointer");
    if (s->device != c->impl->m->device)
      invalid("mlb_decode_sample: the sampler is on another device than the context");
    validate_sampling(c->impl->m->cfg.vocab_size, temperature, top_k);
    context_decode_sample(*c->impl, s->state.as<MtState>(), s->out.as<int>(),
                          s->status.as<DeviceStatus>(), temperature, top_k, token, pos, n_steps,
                          tokens_host);
    check_sampler_status(s);
  });
}

int mlb_decode_greedy(mlb_context* c, int token, int pos, int n_steps, int* tokens_host) {
  return guarded([&] {
    if (!c || (n_steps > 0 && !tokens_host)) invalid("mlb_decode_greedy: null pointer");
    context_decode_greedy(*c->impl, token, pos, n_steps, tokens_host);
  });
}

void* mlb_context_stream(mlb_context* c) { return c ? c->impl->stream : nullptr; }

int mlb_context_kernels_per_step(const mlb_context* c) {
  return c ? c->impl->kernels_per_step : 0;
}

int mlb_context_set_step_kernel(mlb_context* c, int enable) {
  return guarded([&] {
    if (!c) invalid("mlb_context_set_step_kernel: null context");
    c->impl->set_use_step(enable != 0);
  });
}

int mlb_context_step_kernel(const mlb_context* c) { return c && c->impl->use_step ? 1 : 0; }

int mlb_context_step_trace(mlb_context* c, int enable) {
  return guarded([&] {
    if (!c) invalid("mlb_context_step_trace: null context");
    c->impl->set_step_trace(enable != 0);
  });
}

int mlb_context_step_trace_read(mlb_context* c, uint64_t* stamps, size_t cap, int* nphases,
                                int* grid) {
  return guarded([&] {
    if (!c || !nphases || !grid) invalid("mlb_context_step_trace_read: null argument");
    c->impl->read_step_trace(reinterpret_cast<unsigned long long*>(stamps), cap, nphases, grid);
  });
}

int mlb_wait_selftest(int device, int which, double limit_ms, int* code, int* where) {
  return guarded([&] {
    if (!code || !where) invalid("mlb_wait_selftest: null output");
    if (which != 0 && which != 1) invalid("mlb_wait_selftest: which must be 0 or 1");
    if (!(limit_ms > 0.0) || limit_ms > 1000.0)
      invalid("mlb_wait_selftest: limit_ms must be in (0, 1000]");
    set_device(device);
    int khz = 0;
    MLB_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device));
    const long long cycles = (long long)(limit_ms * (double)khz);
    step_wait_selftest(which, cycles > 0 ? cycles : 1, 900 + which, code, where);
  });
}

int mlb_nccl_unique_id(void* out128) {
  return guarded([&] {
    if (!out128) invalid("mlb_nccl_unique_id: null output");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) fail(MLB_ERR_NCCL, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
    std::memcpy(out128, &id, sizeof(id));
  });
}

}  // extern "C"

// ----------------------------------------------------- batches (batch.cu)

namespace mlb {
struct BatchImpl;
BatchImpl* batch_create(ModelImpl& m, int n_seqs, int mode, int kv_type);
void batch_destroy(BatchImpl* b);
void batch_reset(BatchImpl& b);
void batch_fill_kv(BatchImpl& b, int seq, int n_pos, uint64_t seed, float scale);
void batch_forward(BatchImpl& b, int n, const int* seqs, const int* toks, const int* poss,
                   float* logits_host, int* next_host);
void batch_decode_greedy(BatchImpl& b, const int* toks, const int* poss, int steps, int* out_host);
void context_forward_batch(ContextImpl& c, int n, const int* toks, const int* poss,
                           float* logits_host);
int batch_kernels_per_step(const BatchImpl& b);
cudaStream_t batch_stream(const BatchImpl& b);
}  // namespace mlb

struct mlb_batch {
  BatchImpl* impl;
};

int mlb_forward_batch(mlb_context* c, int n_tokens, const int* tokens, const int* positions,
                      float* logits_host) {
  return guarded([&] {
    if (!c || !tokens || !positions || !logits_host) invalid("ForwardBatch: null pointer");
    context_forward_batch(*c->impl, n_tokens, tokens, positions, logits_host);
  });
}

int mlb_batch_create(mlb_model* m, int n_seqs, int attention_mode, mlb_batch** out) {
  return guarded([&] {
    if (!m || !out) invalid("mlb_batch_create: null pointer");
    BatchImpl* b = batch_create(*m->impl, n_seqs, attention_mode, MLB_KV_F32);
    *out = new mlb_batch{b};
  });
}

int mlb_batch_create_kv(mlb_model* m, int n_seqs, int attention_mode, int kv_type,
                        mlb_batch** out) {
  return guarded([&] {
    if (!m || !out) invalid("mlb_batch_create: null pointer");
    BatchImpl* b = batch_create(*m->impl, n_seqs, attention_mode, kv_type);
    *out = new mlb_batch{b};
  });
}

int mlb_batch_destroy(mlb_batch* b) {
  return guarded([&] {
    if (b) {
      batch_destroy(b->impl);
      delete b;
    }
  });
}

int mlb_batch_reset(mlb_batch* b) {
  return guarded([&] {
    if (!b) invalid("mlb_batch_reset: null batch");
    batch_reset(*b->impl);
  });
}

int mlb_batch_fill_kv(mlb_batch* b, int seq, int n_pos, uint64_t seed, float scale) {
  return guarded([&] {
    if (!b) invalid("mlb_batch_fill_kv: null batch");
    batch_fill_kv(*b->impl, seq, n_pos, seed, scale);
  });
}

int mlb_batch_forward(mlb_batch* b, int n_rows, const int* seq_ids, const int* tokens,
                      const int* positions, float* logits_host, int* next_tokens_host) {
  return guarded([&] {
    if (!b || !seq_ids || !tokens || !positions) invalid("mlb_batch_forward: null pointer");
    batch_forward(*b->impl, n_rows, seq_ids, tokens, positions, logits_host, next_tokens_host);
  });
}

int mlb_batch_decode_greedy(mlb_batch* b, const int* tokens, const int* positions, int n_steps,
                            int* tokens_out) {
  return guarded([&] {
    if (!b || !tokens || !positions || !tokens_out) invalid("mlb_batch_decode_greedy: null pointer");
    batch_decode_greedy(*b->impl, tokens, positions, n_steps, tokens_out);
  });
}

void* mlb_batch_stream(mlb_batch* b) { return b ? (void*)batch_stream(*b->impl) : nullptr; }

int mlb_batch_kernels_per_step(const mlb_batch* b) {
  return b ? batch_kernels_per_step(*b->impl) : 0;
}

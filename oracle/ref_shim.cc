// ref_shim.cc — C entry points over the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with
// the reference's unmodified sources (read in place from the reference tree)
// into oracle/_ref/libmlref.so. Tests use it to pin the C restatement in
// oracle/port against the reference itself, and bench.py's reference arm and
// cpu_baseline leg use it to time the reference CPU path. Every entry point
// here calls the reference's public C++ API: LinearQ80/Q40/Q41 and Linear
// (include/mini_llama/ops.h, quant.h), Dequantize*/Quantize* (quant.h),
// RmsNorm/Softmax/SwiGlu/Rope/ArgMax (ops.h), and ForwardToken on a
// MiniLlamaModel with cuda_weights == nullptr (forward.h:11) and SetThreadCount
// (thread_pool.h:10).
#include "mini_llama/context.h"
#include "mini_llama/forward.h"
#include "mini_llama/model.h"
#include "mini_llama/ops.h"
#include "mini_llama/quant.h"
#include "mini_llama/thread_pool.h"

#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

using namespace mini_llama;

namespace {
thread_local std::string g_err;

int Fail(const std::exception& e) {
  g_err = e.what();
  return dynamic_cast<const std::out_of_range*>(&e) ? -2 : -1;
}

Tensor MakeTensor(const float* data, const std::vector<int>& shape) {
  Tensor t(shape, 0.0f);
  if (data) std::memcpy(t.data.data(), data, t.data.size() * sizeof(float));
  return t;
}

QuantizedTensor MakeQuantized(int qtype, int rows, int cols, const void* data) {
  QuantizedTensor q;
  q.shape = {rows, cols};
  size_t nb = static_cast<size_t>(rows) * ((cols + 31) / 32);
  switch (qtype) {
    case 0:
      q.type = QuantType::kF32;
      q.f32_data.resize(static_cast<size_t>(rows) * cols);
      std::memcpy(q.f32_data.data(), data, q.f32_data.size() * sizeof(float));
      break;
    case 1:
      q.type = QuantType::kQ80;
      q.q8_0_data.resize(nb);
      std::memcpy(q.q8_0_data.data(), data, nb * sizeof(BlockQ80));
      break;
    case 2:
      q.type = QuantType::kQ40;
      q.q4_0_data.resize(nb);
      std::memcpy(q.q4_0_data.data(), data, nb * sizeof(BlockQ40));
      break;
    case 3:
      q.type = QuantType::kQ41;
      q.q4_1_data.resize(nb);
      std::memcpy(q.q4_1_data.data(), data, nb * sizeof(BlockQ41));
      break;
    default:
      throw std::runtime_error("ref shim: unsupported quant type");
  }
  return q;
}

struct RefModel {
  MiniLlamaModel model;
};
struct RefCtx {
  RefModel* m;
  std::unique_ptr<MiniLlamaContext> ctx;
};
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

void ref_set_threads(int n) { SetThreadCount(n); }
int ref_get_threads(void) { return GetThreadCount(); }

int ref_linear(int qtype, const float* x, int rows, int in_features,
               const void* w, int out_features, float* y) {
  try {
    Tensor xt = rows == 1 ? MakeTensor(x, {in_features})
                          : MakeTensor(x, {rows, in_features});
    QuantizedTensor q = MakeQuantized(qtype, out_features, in_features, w);
    Tensor out = Linear(xt, q);
    std::memcpy(y, out.data.data(), out.data.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_dequant(int qtype, const void* w, int rows, int cols, float* out) {
  try {
    QuantizedTensor q = MakeQuantized(qtype, rows, cols, w);
    Tensor t;
    switch (qtype) {
      case 1: t = DequantizeFromQ80(q.q8_0_data, q.shape); break;
      case 2: t = DequantizeFromQ40(q.q4_0_data, q.shape); break;
      case 3: t = DequantizeFromQ41(q.q4_1_data, q.shape); break;
      default: t = ToTensor(q); break;
    }
    std::memcpy(out, t.data.data(), t.data.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_quantize(int qtype, const float* src, int rows, int cols, void* out) {
  try {
    Tensor t = MakeTensor(src, {rows, cols});
    if (qtype == 1) {
      auto b = QuantizeToQ80(t);
      std::memcpy(out, b.data(), b.size() * sizeof(BlockQ80));
    } else if (qtype == 2) {
      auto b = QuantizeToQ40(t);
      std::memcpy(out, b.data(), b.size() * sizeof(BlockQ40));
    } else {
      throw std::runtime_error("ref_quantize: only Q8_0 and Q4_0 have a reference quantizer");
    }
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_rmsnorm(const float* x, const float* w, int n, float eps, float* y) {
  try {
    Tensor out = RmsNorm(MakeTensor(x, {n}), MakeTensor(w, {n}), eps);
    std::memcpy(y, out.data.data(), n * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_softmax(const float* x, int n, float* y) {
  try {
    Tensor out = Softmax(MakeTensor(x, {n}));
    std::memcpy(y, out.data.data(), n * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_swiglu(const float* g, const float* u, int n, float* y) {
  try {
    Tensor out = SwiGlu(MakeTensor(g, {n}), MakeTensor(u, {n}));
    std::memcpy(y, out.data.data(), n * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_rope(float* q, int n_heads, float* k, int n_kv_heads, int head_dim,
             int pos, float theta, int neox) {
  try {
    Tensor qt = MakeTensor(q, {n_heads, head_dim});
    Tensor kt = MakeTensor(k, {n_kv_heads, head_dim});
    Rope(qt, kt, pos, theta, neox ? RopeType::kNeoX : RopeType::kNormal);
    std::memcpy(q, qt.data.data(), qt.data.size() * sizeof(float));
    std::memcpy(k, kt.data.data(), kt.data.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_argmax(const float* x, int n) {
  try {
    return ArgMax(MakeTensor(x, {n}));
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

// ---- model ---------------------------------------------------------------

void* ref_model_create(int vocab_size, int dim, int hidden_dim, int n_layers,
                       int n_heads, int n_kv_heads, int head_dim,
                       int max_seq_len, float rope_theta, float rms_norm_eps,
                       int rope_type) {
  auto* m = new RefModel();
  ModelConfig& c = m->model.config;
  c.vocab_size = vocab_size;
  c.dim = dim;
  c.hidden_dim = hidden_dim;
  c.n_layers = n_layers;
  c.n_heads = n_heads;
  c.n_kv_heads = n_kv_heads;
  c.head_dim = head_dim;
  c.max_seq_len = max_seq_len;
  c.rope_theta = rope_theta;
  c.rms_norm_eps = rms_norm_eps;
  c.rope_type = rope_type ? RopeType::kNeoX : RopeType::kNormal;
  m->model.layers.resize(n_layers);
  m->model.loaded = true;
  return m;
}

void ref_model_destroy(void* h) { delete static_cast<RefModel*>(h); }

// kind follows the upload order of src/model.cc:353-369.
int ref_model_set_weight(void* h, int kind, int layer, int qtype, int rows,
                         int cols, const void* data) {
  try {
    MiniLlamaModel& m = static_cast<RefModel*>(h)->model;
    auto f32 = [&](bool one_d) {
      return one_d ? MakeTensor(static_cast<const float*>(data), {rows * cols})
                   : MakeTensor(static_cast<const float*>(data), {rows, cols});
    };
    if (kind == 0) { m.token_embedding = f32(false); return 0; }
    if (kind == 1) { m.final_norm = f32(true); return 0; }
    if (kind == 2) { m.lm_head = MakeQuantized(qtype, rows, cols, data); return 0; }
    if (layer < 0 || layer >= static_cast<int>(m.layers.size()))
      throw std::out_of_range("ref_model_set_weight: layer out of range");
    LayerWeights& lw = m.layers[layer];
    switch (kind) {
      case 3: lw.attention_norm = f32(true); break;
      case 4: lw.wq = MakeQuantized(qtype, rows, cols, data); break;
      case 5: lw.wk = MakeQuantized(qtype, rows, cols, data); break;
      case 6: lw.wv = MakeQuantized(qtype, rows, cols, data); break;
      case 7: lw.bq = f32(true); break;
      case 8: lw.bk = f32(true); break;
      case 9: lw.bv = f32(true); break;
      case 10: lw.wo = MakeQuantized(qtype, rows, cols, data); break;
      case 11: lw.ffn_norm = f32(true); break;
      case 12: lw.w_gate = MakeQuantized(qtype, rows, cols, data); break;
      case 13: lw.w_up = MakeQuantized(qtype, rows, cols, data); break;
      case 14: lw.w_down = MakeQuantized(qtype, rows, cols, data); break;
      default: throw std::out_of_range("ref_model_set_weight: kind out of range");
    }
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

int ref_model_config(void* h, int* out11) {
  const ModelConfig& c = static_cast<RefModel*>(h)->model.config;
  int v[11] = {c.vocab_size, c.dim, c.hidden_dim, c.n_layers, c.n_heads,
               c.n_kv_heads, c.head_dim, c.max_seq_len, 0, 0,
               c.rope_type == RopeType::kNeoX ? 1 : 0};
  std::memcpy(out11, v, sizeof(v));
  return 0;
}

void* ref_ctx_create(void* h) {
  try {
    auto* c = new RefCtx();
    c->m = static_cast<RefModel*>(h);
    c->ctx = std::make_unique<MiniLlamaContext>(&c->m->model);
    return c;
  } catch (const std::exception& e) {
    Fail(e);
    return nullptr;
  }
}

void ref_ctx_destroy(void* c) { delete static_cast<RefCtx*>(c); }

// ForwardToken (CPU branch: the model has no cuda_weights).
int ref_forward_token(void* ch, int token, int pos, float* logits) {
  try {
    auto* c = static_cast<RefCtx*>(ch);
    c->ctx->pos = pos;
    Tensor out = ForwardToken(*c->ctx, c->m->model, token);
    std::memcpy(logits, out.data.data(), out.data.size() * sizeof(float));
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

}  // extern "C"

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
// MiniLlamaModel with cuda_weights == nullptr (forward.h:11), SetThreadCount
// (thread_pool.h:10), MiniSampler (sampler.h) and LoadGgufModel
// (gguf_loader.h).
#include "mini_llama/context.h"
#include "mini_llama/forward.h"
#include "mini_llama/gguf_loader.h"
#include "mini_llama/model.h"
#include "mini_llama/ops.h"
#include "mini_llama/quant.h"
#include "mini_llama/sampler.h"
#include "mini_llama/thread_pool.h"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <exception>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "synth.h"  // the seeded input generator shared with the GPU library

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

// LoadGgufModel (src/gguf_loader.cc:302-418) on a GGUF file; null (with the
// model's load_error as the message) when the reference refuses the file.
void* ref_model_load_gguf(const char* path) {
  try {
    auto m = std::make_unique<RefModel>();
    m->model = LoadGgufModel(path);
    if (!m->model.loaded) {
      g_err = m->model.load_error;
      return nullptr;
    }
    return m.release();
  } catch (const std::exception& e) {
    Fail(e);
    return nullptr;
  }
}

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

// Every weight of the model from the seeded generator (synth.h, the same
// definition the GPU library generates from): fp32 values gauss(key, index) *
// 0.02, quantised here with the reference's own QuantizeToQ80 / QuantizeToQ40
// (src/quant.cc:106-276); Q4_1 has no quantiser in the reference's library,
// so it takes the generator's restatement of the reference test's
// QuantizeToQ41ForTest. Norms are 1.0, the embedding fp32, biases (when
// with_bias) fp32. Rows are generated and quantised in chunks on `threads`
// threads, so no full fp32 copy of a large matrix is ever held. The bytes equal
// what the GPU library's generator writes (the tests compare them).
int ref_model_synthesize(void* h, int qtype, uint64_t seed, int with_bias, int threads) {
  try {
    MiniLlamaModel& m = static_cast<RefModel*>(h)->model;
    const ModelConfig& c = m.config;
    if (qtype < 1 || qtype > 3) throw std::runtime_error("ref_model_synthesize: quantised types only");
    threads = threads < 1 ? 1 : threads;
    auto key_of = [&](int kind, int layer) {
      return mlb::synth::stream_key(seed, (uint64_t)kind * (1ull << 20) + (uint64_t)(layer < 0 ? 0 : layer));
    };
    auto par = [&](long long rows, const std::function<void(long long, long long)>& f) {
      const long long chunk = 64;
      const long long nchunks = (rows + chunk - 1) / chunk;
      std::atomic<long long> next{0};
      std::vector<std::thread> ts;
      std::exception_ptr err;
      std::mutex mu;
      for (int t = 0; t < threads; ++t)
        ts.emplace_back([&] {
          try {
            for (long long i; (i = next.fetch_add(1)) < nchunks;)
              f(i * chunk, std::min(rows, (i + 1) * chunk));
          } catch (...) {
            std::lock_guard<std::mutex> g(mu);
            err = std::current_exception();
          }
        });
      for (auto& th : ts) th.join();
      if (err) std::rethrow_exception(err);
    };
    auto f32 = [&](int kind, int layer, int rows, int cols, bool one_d) {
      Tensor t(one_d ? std::vector<int>{rows * cols} : std::vector<int>{rows, cols}, 0.0f);
      const uint64_t key = key_of(kind, layer);
      par(rows, [&](long long a, long long b) {
        for (long long r = a; r < b; ++r)
          for (int j = 0; j < cols; ++j)
            t.data[(size_t)r * cols + j] =
                mlb::synth::fmul(mlb::synth::gauss(key, (uint64_t)(r * cols + j)), 0.02f);
      });
      return t;
    };
    auto ones = [&](int n) { return Tensor(std::vector<int>{n}, 1.0f); };
    auto quant = [&](int kind, int layer, int rows, int cols) {
      QuantizedTensor q;
      q.shape = {rows, cols};
      const int nb = (cols + 31) / 32;
      const uint64_t key = key_of(kind, layer);
      const size_t nblk = (size_t)rows * nb;
      if (qtype == 1) { q.type = QuantType::kQ80; q.q8_0_data.resize(nblk); }
      if (qtype == 2) { q.type = QuantType::kQ40; q.q4_0_data.resize(nblk); }
      if (qtype == 3) { q.type = QuantType::kQ41; q.q4_1_data.resize(nblk); }
      par(rows, [&](long long a, long long b) {
        Tensor src(std::vector<int>{(int)(b - a), cols}, 0.0f);
        for (long long r = a; r < b; ++r)
          for (int j = 0; j < cols; ++j)
            src.data[(size_t)(r - a) * cols + j] =
                mlb::synth::fmul(mlb::synth::gauss(key, (uint64_t)(r * cols + j)), 0.02f);
        const size_t off = (size_t)a * nb;
        if (qtype == 1) {
          auto blk = QuantizeToQ80(src);
          std::memcpy(&q.q8_0_data[off], blk.data(), blk.size() * sizeof(BlockQ80));
        } else if (qtype == 2) {
          auto blk = QuantizeToQ40(src);
          std::memcpy(&q.q4_0_data[off], blk.data(), blk.size() * sizeof(BlockQ40));
        } else {
          for (long long r = a; r < b; ++r)
            for (int j = 0; j < nb; ++j) {
              const int n = std::min(32, cols - 32 * j);
              mlb::synth::quantize_q4_1(&src.data[(size_t)(r - a) * cols + 32 * j], n,
                                        reinterpret_cast<uint8_t*>(&q.q4_1_data[(size_t)r * nb + j]));
            }
        }
      });
      return q;
    };
    const int D = c.head_dim, qd = c.n_heads * D, kvd = c.n_kv_heads * D;
    for (int l = 0; l < c.n_layers; ++l) {
      LayerWeights& lw = m.layers[l];
      lw.attention_norm = ones(c.dim);
      lw.wq = quant(4, l, qd, c.dim);
      lw.wk = quant(5, l, kvd, c.dim);
      lw.wv = quant(6, l, kvd, c.dim);
      if (with_bias) {
        lw.bq = f32(7, l, 1, qd, true);
        lw.bk = f32(8, l, 1, kvd, true);
        lw.bv = f32(9, l, 1, kvd, true);
      }
      lw.wo = quant(10, l, c.dim, qd);
      lw.ffn_norm = ones(c.dim);
      lw.w_gate = quant(12, l, c.hidden_dim, c.dim);
      lw.w_up = quant(13, l, c.hidden_dim, c.dim);
      lw.w_down = quant(14, l, c.dim, c.hidden_dim);
    }
    m.token_embedding = f32(0, -1, c.vocab_size, c.dim, false);
    m.final_norm = ones(c.dim);
    m.lm_head = quant(2, -1, c.vocab_size, c.dim);
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
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

// Positions [0, n_pos) of every layer's K and V rows from the seeded
// generator, written through the reference's own KvCache::Write
// (src/kv_cache.cc): element (pos, kv_head, d) of layer l is
// gauss(key, (pos * n_kv_heads + kv_head) * head_dim + d) * scale with the keys
// of streams 15 * 2^20 + l (K) and 16 * 2^20 + l (V). The GPU library's
// mlb_context_fill_kv writes the same values, so both decode from the same
// state at depth n_pos.
int ref_ctx_fill_kv(void* ch, int n_pos, uint64_t seed, float scale) {
  try {
    auto* c = static_cast<RefCtx*>(ch);
    const ModelConfig& cf = c->m->model.config;
    if (n_pos < 0 || n_pos > cf.max_seq_len) throw std::out_of_range("ref_ctx_fill_kv: n_pos out of range");
    const int KV = cf.n_kv_heads, D = cf.head_dim;
    Tensor k(std::vector<int>{KV, D}, 0.0f), v(std::vector<int>{KV, D}, 0.0f);
    for (int l = 0; l < cf.n_layers; ++l) {
      const uint64_t kk = mlb::synth::stream_key(seed, 15ull * (1ull << 20) + (uint64_t)l);
      const uint64_t kv = mlb::synth::stream_key(seed, 16ull * (1ull << 20) + (uint64_t)l);
      for (int p = 0; p < n_pos; ++p) {
        for (int i = 0; i < KV * D; ++i) {
          const uint64_t idx = (uint64_t)p * KV * D + (uint64_t)i;
          k.data[i] = mlb::synth::fmul(mlb::synth::gauss(kk, idx), scale);
          v.data[i] = mlb::synth::fmul(mlb::synth::gauss(kv, idx), scale);
        }
        c->ctx->kv_cache.Write(l, p, k, v);
      }
    }
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

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

// MiniSampler(seed) and MiniSampler::Sample (src/sampler.cc:89-183).
void* ref_sampler_create(unsigned int seed) {
  try {
    return new MiniSampler(seed);
  } catch (const std::exception& e) {
    Fail(e);
    return nullptr;
  }
}

void ref_sampler_destroy(void* s) { delete static_cast<MiniSampler*>(s); }

int ref_sample(void* s, const float* logits, int n, float temperature, int top_k, int* out) {
  try {
    Tensor t(std::vector<int>{n});
    std::memcpy(t.data.data(), logits, (size_t)n * sizeof(float));
    SamplingParams p;
    p.temperature = temperature;
    p.top_k = top_k;
    *out = static_cast<MiniSampler*>(s)->Sample(t, p);
    return 0;
  } catch (const std::exception& e) {
    return Fail(e);
  }
}

}  // extern "C"

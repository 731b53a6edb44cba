/*
 * mlport.c — CPU restatement of the reference's decode forward path.
 *
 * TEST INFRASTRUCTURE ONLY (the oracle). See mlport.h for the contract.
 * Build with -ffp-contract=off: every product and sum is rounded on its own,
 * as in the reference's x86-64 build (which has no FMA contraction).
 */
#include "mlport.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

static __thread char g_err[512];

static int fail(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

const char* mlp_last_error(void) { return g_err; }

/* GGUF block layouts, include/mini_llama/quantized_tensor.h:26-44. */
typedef struct {
  uint16_t d;
  int8_t qs[32];
} blk_q8_0; /* 34 bytes */
typedef struct {
  uint16_t d;
  uint8_t qs[16];
} blk_q4_0; /* 18 bytes */
typedef struct {
  uint16_t d;
  uint16_t m;
  uint8_t qs[16];
} blk_q4_1; /* 20 bytes */

_Static_assert(sizeof(blk_q8_0) == 34, "Q8_0 block is 34 bytes");
_Static_assert(sizeof(blk_q4_0) == 18, "Q4_0 block is 18 bytes");
_Static_assert(sizeof(blk_q4_1) == 20, "Q4_1 block is 20 bytes");

/* Exact binary16 -> binary32 widening; src/quant.cc:53-84. */
float mlp_fp16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      /* subnormal: shift the leading one up to the implicit-bit position */
      int shifts = 0;
      while ((m & 0x400u) == 0) {
        m <<= 1;
        ++shifts;
      }
      bits = sign | ((uint32_t)(113 - shifts) << 23) | ((m & 0x3ffu) << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  float out;
  memcpy(&out, &bits, sizeof(out));
  return out;
}

/*
 * binary32 -> binary16 with the reference's rounding: the dropped part is
 * rounded half-up on its top bit (not ties-to-even); src/quant.cc:14-50.
 */
uint16_t mlp_f32_to_fp16(float f) {
  uint32_t b;
  memcpy(&b, &f, sizeof(b));
  uint32_t sign = (b >> 16) & 0x8000u;
  int32_t e = (int32_t)((b >> 23) & 0xffu) - 112;
  uint32_t m = b & 0x7fffffu;
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    uint32_t s = (m | 0x800000u) >> (1 - e);
    if (s & 0x1000u) s += 0x2000u;
    return (uint16_t)(sign | (s >> 13));
  }
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (m & 0x1000u) {
    m += 0x2000u;
    if (m & 0x800000u) {
      m = 0;
      if (++e >= 31) return (uint16_t)(sign | 0x7c00u);
    }
  }
  return (uint16_t)(sign | ((uint32_t)e << 10) | (m >> 13));
}

size_t mlp_block_bytes(int qtype) {
  switch (qtype) {
    case MLP_F32: return 4;
    case MLP_Q8_0: return sizeof(blk_q8_0);
    case MLP_Q4_0: return sizeof(blk_q4_0);
    case MLP_Q4_1: return sizeof(blk_q4_1);
  }
  return 0;
}

size_t mlp_weight_bytes(int qtype, int rows, int cols) {
  if (qtype == MLP_F32) return (size_t)rows * (size_t)cols * 4u;
  size_t nb = (size_t)((cols + 31) / 32);
  return (size_t)rows * nb * mlp_block_bytes(qtype);
}

/* One dequantised element; src/quant.cc:430-456. */
static inline float dq_q8_0(const blk_q8_0* b, int i) {
  return mlp_fp16_to_f32(b->d) * (float)b->qs[i];
}
static inline float dq_q4_0(const blk_q4_0* b, int i) {
  int q = i < 16 ? (int)(b->qs[i] & 0x0f) - 8 : (int)(b->qs[i - 16] >> 4) - 8;
  return mlp_fp16_to_f32(b->d) * (float)q;
}
static inline float dq_q4_1(const blk_q4_1* b, int i) {
  int q = i < 16 ? (int)(b->qs[i] & 0x0f) : (int)(b->qs[i - 16] >> 4);
  return mlp_fp16_to_f32(b->d) * (float)q + mlp_fp16_to_f32(b->m);
}

static float dq_elem(int qtype, const void* w, size_t block, int i) {
  switch (qtype) {
    case MLP_Q8_0: return dq_q8_0((const blk_q8_0*)w + block, i);
    case MLP_Q4_0: return dq_q4_0((const blk_q4_0*)w + block, i);
    default: return dq_q4_1((const blk_q4_1*)w + block, i);
  }
}

/* DequantizeFromQ80/Q40/Q41, src/quant.cc:170-361 (row-wise, tail-padded). */
int mlp_dequant(int qtype, const void* w, int rows, int cols, float* out) {
  if (rows < 0 || cols < 0) return fail(-1, "mlp_dequant: negative shape");
  if (qtype == MLP_F32) {
    memcpy(out, w, (size_t)rows * (size_t)cols * 4u);
    return 0;
  }
  int nb = (cols + 31) / 32;
  for (int r = 0; r < rows; ++r)
    for (int b = 0; b < nb; ++b)
      for (int i = 0; i < 32 && b * 32 + i < cols; ++i)
        out[(size_t)r * cols + b * 32 + i] =
            dq_elem(qtype, w, (size_t)r * nb + b, i);
  return 0;
}

static void quant_block_q8_0(const float* x, int n, blk_q8_0* out) {
  /* QuantizeToQ80, src/quant.cc:106-167: d = absmax/127, q = round(x/d). */
  memset(out, 0, sizeof(*out));
  float amax = 0.0f;
  for (int i = 0; i < n; ++i) {
    float a = fabsf(x[i]);
    if (a > amax) amax = a;
  }
  if (!(amax > 0.0f)) return;
  out->d = mlp_f32_to_fp16(amax / 127.0f);
  float sd = mlp_fp16_to_f32(out->d);
  float inv = sd == 0.0f ? 0.0f : 1.0f / sd;
  for (int i = 0; i < n; ++i) {
    int q = (int)roundf(x[i] * inv);
    if (q > 127) q = 127;
    if (q < -127) q = -127;
    out->qs[i] = (int8_t)q;
  }
}

static void quant_block_q4_0(const float* x, int n, blk_q4_0* out) {
  /* QuantizeToQ40, src/quant.cc:201-276: d = absmax/7, q = round(x/d + 8). */
  memset(out, 0, sizeof(*out));
  float amax = 0.0f;
  for (int i = 0; i < n; ++i) {
    float a = fabsf(x[i]);
    if (a > amax) amax = a;
  }
  if (!(amax > 0.0f)) return;
  out->d = mlp_f32_to_fp16(amax / 7.0f);
  float sd = mlp_fp16_to_f32(out->d);
  float inv = sd == 0.0f ? 0.0f : 1.0f / sd;
  for (int j = 0; j < 16; ++j) {
    float v0 = j < n ? x[j] * inv : 0.0f;
    float v1 = j + 16 < n ? x[j + 16] * inv : 0.0f;
    int q0 = (int)roundf(v0 + 8.0f);
    int q1 = (int)roundf(v1 + 8.0f);
    q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
    q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
    out->qs[j] = (uint8_t)(q0 | (q1 << 4));
  }
}

static void quant_block_q4_1(const float* x, int n, blk_q4_1* out) {
  /*
   * The reference has no production Q4_1 quantizer; its tests use
   * QuantizeToQ41ForTest, tests/test_cuda_quant.cc:131-188:
   * d = (max - min)/15, m = min, q = round((x - m)/d).
   */
  memset(out, 0, sizeof(*out));
  float lo = INFINITY, hi = -INFINITY;
  for (int i = 0; i < n; ++i) {
    if (x[i] < lo) lo = x[i];
    if (x[i] > hi) hi = x[i];
  }
  float range = hi - lo;
  if (range > 0.0f) {
    out->d = mlp_f32_to_fp16(range / 15.0f);
    out->m = mlp_f32_to_fp16(lo);
    float sd = mlp_fp16_to_f32(out->d);
    float sm = mlp_fp16_to_f32(out->m);
    float inv = sd == 0.0f ? 0.0f : 1.0f / sd;
    for (int j = 0; j < 16; ++j) {
      int q0 = j < n ? (int)roundf((x[j] - sm) * inv) : 0;
      int q1 = j + 16 < n ? (int)roundf((x[j + 16] - sm) * inv) : 0;
      q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
      q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
      out->qs[j] = (uint8_t)(q0 | (q1 << 4));
    }
  } else {
    out->m = mlp_f32_to_fp16(lo == INFINITY ? 0.0f : lo);
  }
}

int mlp_quantize(int qtype, const float* src, int rows, int cols, void* out) {
  if (rows < 0 || cols < 0) return fail(-1, "mlp_quantize: negative shape");
  int nb = (cols + 31) / 32;
  for (int r = 0; r < rows; ++r) {
    for (int b = 0; b < nb; ++b) {
      const float* x = src + (size_t)r * cols + b * 32;
      int n = cols - b * 32 < 32 ? cols - b * 32 : 32;
      size_t bi = (size_t)r * nb + b;
      switch (qtype) {
        case MLP_Q8_0: quant_block_q8_0(x, n, (blk_q8_0*)out + bi); break;
        case MLP_Q4_0: quant_block_q4_0(x, n, (blk_q4_0*)out + bi); break;
        case MLP_Q4_1: quant_block_q4_1(x, n, (blk_q4_1*)out + bi); break;
        default: return fail(-1, "mlp_quantize: unsupported type");
      }
    }
  }
  return 0;
}

/*
 * y[r, j] = sum_k w[j, k] * x[r, k], one sequential fp32 sum per output in
 * block order; LinearQuantizedImpl, src/quant.cc:365-425 (quantised) and
 * LinearThreaded, src/matmul_optimized.cc:73-91 (F32, x times w order).
 */
int mlp_linear(int qtype, const float* x, int rows, int in_features,
               const void* w, int out_features, float* y) {
  if (rows <= 0 || in_features <= 0 || out_features <= 0)
    return fail(-1, "mlp_linear: empty tensors are not supported");
  if (qtype == MLP_F32) {
    const float* wf = (const float*)w;
    for (int r = 0; r < rows; ++r) {
      const float* xr = x + (size_t)r * in_features;
      for (int j = 0; j < out_features; ++j) {
        float s = 0.0f;
        const float* wr = wf + (size_t)j * in_features;
        for (int k = 0; k < in_features; ++k) s += xr[k] * wr[k];
        y[(size_t)r * out_features + j] = s;
      }
    }
    return 0;
  }
  if (qtype != MLP_Q8_0 && qtype != MLP_Q4_0 && qtype != MLP_Q4_1)
    return fail(-1, "mlp_linear: unsupported type");
  int nb = (in_features + 31) / 32;
  for (int r = 0; r < rows; ++r) {
    const float* xr = x + (size_t)r * in_features;
    for (int j = 0; j < out_features; ++j) {
      float s = 0.0f;
      for (int b = 0; b < nb; ++b) {
        size_t bi = (size_t)j * nb + b;
        int k_end = b * 32 + 32 < in_features ? b * 32 + 32 : in_features;
        for (int k = b * 32; k < k_end; ++k)
          s += dq_elem(qtype, w, bi, k - b * 32) * xr[k];
      }
      y[(size_t)r * out_features + j] = s;
    }
  }
  return 0;
}

/* RmsNorm, src/ops.cc:43-68: y = (x * 1/sqrt(mean(x^2) + eps)) * w. */
void mlp_rmsnorm(const float* x, const float* w, int n, float eps, float* y) {
  float ss = 0.0f;
  for (int i = 0; i < n; ++i) ss += x[i] * x[i];
  ss /= (float)n;
  float scale = 1.0f / sqrtf(ss + eps);
  for (int i = 0; i < n; ++i) y[i] = x[i] * scale * w[i];
}

/* Softmax, src/ops.cc:71-98. */
void mlp_softmax(const float* x, int n, float* y) {
  float mx = x[0];
  for (int i = 1; i < n; ++i)
    if (mx < x[i]) mx = x[i];
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    y[i] = expf(x[i] - mx);
    sum += y[i];
  }
  for (int i = 0; i < n; ++i) y[i] /= sum;
}

/* SwiGlu, src/ops.cc:128-140: (g * sigmoid(g)) * u. */
void mlp_swiglu(const float* gate, const float* up, int n, float* y) {
  for (int i = 0; i < n; ++i) {
    float g = gate[i];
    float sg = 1.0f / (1.0f + expf(-g));
    y[i] = g * sg * up[i];
  }
}

/*
 * Rope, src/ops.cc:143-216. Normal RoPE rotates (2i, 2i+1) by
 * pos * theta^(-2i/D); NeoX rotates (i, i + D/2) by pos * theta^(-2i/D).
 */
static void rope_heads(float* x, int heads, int d, int pos, float theta,
                       int neox) {
  for (int h = 0; h < heads; ++h) {
    float* v = x + (size_t)h * d;
    if (!neox) {
      for (int i = 0; i < d; i += 2) {
        float freq = 1.0f / powf(theta, (float)i / (float)d);
        float c = cosf((float)pos * freq), s = sinf((float)pos * freq);
        float a = v[i], b = v[i + 1];
        v[i] = a * c - b * s;
        v[i + 1] = a * s + b * c;
      }
    } else {
      int half = d / 2;
      for (int i = 0; i < half; ++i) {
        float freq = 1.0f / powf(theta, (float)(2 * i) / (float)d);
        float c = cosf((float)pos * freq), s = sinf((float)pos * freq);
        float a = v[i], b = v[i + half];
        v[i] = a * c - b * s;
        v[i + half] = a * s + b * c;
      }
    }
  }
}

void mlp_rope(float* q, int n_heads, float* k, int n_kv_heads, int head_dim,
              int pos, float theta, int neox) {
  rope_heads(q, n_heads, head_dim, pos, theta, neox);
  rope_heads(k, n_kv_heads, head_dim, pos, theta, neox);
}

/* 1/sqrt(D) evaluated as in src/forward.cc:489 (double quotient, float store). */
float mlp_attention_scale(int head_dim) {
  return (float)(1.0 / (double)sqrtf((float)head_dim));
}

/*
 * Decode attention over the KV cache [L][max_seq][KV][D], GQA head map
 * h / (H/KV); src/forward.cc:487-545 (CPU) with the softmax over t in
 * [0, pos]. The reference CPU path sums V over t < pos only
 * (src/forward.cc:518); include_current_v = 1 sums t <= pos instead, as the
 * reference GPU kernel (src/cuda_attention.cu:194) and its test-side
 * reference (tests/test_cuda_attention.cc:74) do.
 */
void mlp_attention(const float* q, const float* keys, const float* values,
                   int layer, int max_seq_len, int n_heads, int n_kv_heads,
                   int head_dim, int pos, int include_current_v, float* out) {
  float scale = mlp_attention_scale(head_dim);
  int group = n_heads / n_kv_heads;
  size_t pos_stride = (size_t)n_kv_heads * head_dim;
  size_t layer_base = (size_t)layer * max_seq_len * pos_stride;
  float* scores = (float*)malloc(sizeof(float) * (size_t)(pos + 1));
  float* probs = (float*)malloc(sizeof(float) * (size_t)(pos + 1));
  int v_end = include_current_v ? pos + 1 : pos;
  for (int h = 0; h < n_heads; ++h) {
    int kvh = h / group;
    const float* qh = q + (size_t)h * head_dim;
    for (int t = 0; t <= pos; ++t) {
      const float* kp = keys + layer_base + t * pos_stride + (size_t)kvh * head_dim;
      float dot = 0.0f;
      for (int d = 0; d < head_dim; ++d) dot += qh[d] * kp[d];
      scores[t] = dot * scale;
    }
    mlp_softmax(scores, pos + 1, probs);
    for (int d = 0; d < head_dim; ++d) {
      float acc = 0.0f;
      for (int t = 0; t < v_end; ++t)
        acc += probs[t] *
               values[layer_base + t * pos_stride + (size_t)kvh * head_dim + d];
      out[(size_t)h * head_dim + d] = acc;
    }
  }
  free(scores);
  free(probs);
}

/* ArgMax, src/ops.cc:220-233: the lowest index wins ties. */
int mlp_argmax(const float* x, int n) {
  int best = 0;
  float bv = x[0];
  for (int i = 1; i < n; ++i)
    if (x[i] > bv) {
      bv = x[i];
      best = i;
    }
  return best;
}

/* ---------------------------------------------------------------- model */

typedef struct {
  int qtype, rows, cols;
  void* data;
} weight_t;

struct mlp_model {
  mlp_config c;
  weight_t global[3];            /* embedding, final_norm, lm_head */
  weight_t* layer;               /* n_layers * 12 (kinds 3..14) */
};

struct mlp_ctx {
  mlp_model* m;
  float* keys;
  float* values;
  int kv_bf16; /* K and V rounded to bf16 when written (not a reference mode) */
  /* scratch */
  float *x, *h, *q, *k, *v, *att, *proj, *gate, *up, *act;
};

mlp_model* mlp_model_create(const mlp_config* cfg) {
  mlp_model* m = (mlp_model*)calloc(1, sizeof(mlp_model));
  if (!m) return NULL;
  m->c = *cfg;
  m->layer = (weight_t*)calloc((size_t)cfg->n_layers * 12, sizeof(weight_t));
  return m;
}

void mlp_model_destroy(mlp_model* m) {
  if (!m) return;
  for (int i = 0; i < 3; ++i) free(m->global[i].data);
  for (int i = 0; i < m->c.n_layers * 12; ++i) free(m->layer[i].data);
  free(m->layer);
  free(m);
}

static weight_t* slot(mlp_model* m, int kind, int layer) {
  if (kind < 0 || kind >= MLP_W_COUNT) return NULL;
  if (kind < 3) return &m->global[kind];
  if (layer < 0 || layer >= m->c.n_layers) return NULL;
  return &m->layer[layer * 12 + (kind - 3)];
}

int mlp_model_set_weight(mlp_model* m, int kind, int layer, int qtype,
                         int rows, int cols, const void* data, size_t bytes) {
  weight_t* w = slot(m, kind, layer);
  if (!w) return fail(-2, "mlp_model_set_weight: kind or layer out of range");
  if (bytes != mlp_weight_bytes(qtype, rows, cols))
    return fail(-1, "mlp_model_set_weight: byte count mismatch");
  free(w->data);
  w->data = malloc(bytes ? bytes : 1);
  memcpy(w->data, data, bytes);
  w->qtype = qtype;
  w->rows = rows;
  w->cols = cols;
  return 0;
}

mlp_ctx* mlp_ctx_create(mlp_model* m) {
  const mlp_config* c = &m->c;
  mlp_ctx* x = (mlp_ctx*)calloc(1, sizeof(mlp_ctx));
  size_t kv = (size_t)c->n_layers * c->max_seq_len * c->n_kv_heads * c->head_dim;
  x->m = m;
  x->keys = (float*)calloc(kv, sizeof(float));
  x->values = (float*)calloc(kv, sizeof(float));
  size_t qd = (size_t)c->n_heads * c->head_dim;
  size_t kd = (size_t)c->n_kv_heads * c->head_dim;
  x->x = (float*)calloc((size_t)c->dim, 4);
  x->h = (float*)calloc((size_t)c->dim, 4);
  x->q = (float*)calloc(qd, 4);
  x->k = (float*)calloc(kd, 4);
  x->v = (float*)calloc(kd, 4);
  x->att = (float*)calloc(qd, 4);
  x->proj = (float*)calloc((size_t)c->dim, 4);
  x->gate = (float*)calloc((size_t)c->hidden_dim, 4);
  x->up = (float*)calloc((size_t)c->hidden_dim, 4);
  x->act = (float*)calloc((size_t)c->hidden_dim, 4);
  if (!x->keys || !x->values) {
    mlp_ctx_destroy(x);
    return NULL;
  }
  return x;
}

void mlp_ctx_destroy(mlp_ctx* c) {
  if (!c) return;
  free(c->keys);
  free(c->values);
  free(c->x);
  free(c->h);
  free(c->q);
  free(c->k);
  free(c->v);
  free(c->att);
  free(c->proj);
  free(c->gate);
  free(c->up);
  free(c->act);
  free(c);
}

/* x rounded to the nearest bf16 (ties to even), kept as a float: the value a
 * bf16 KV cache stores. Not part of the reference, which keeps fp32 K/V; the
 * switch mirrors the GPU library's bf16 cache option. */
static float bf16_round(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  memcpy(&x, &u, 4);
  return x;
}

void mlp_ctx_set_kv_bf16(mlp_ctx* c, int on) { c->kv_bf16 = on; }

void mlp_ctx_kv(mlp_ctx* c, float** keys, float** values) {
  *keys = c->keys;
  *values = c->values;
}

static int lin(const weight_t* w, const float* x, float* y) {
  return mlp_linear(w->qtype, x, 1, w->cols, w->data, w->rows, y);
}

static void add_bias(float* y, const weight_t* b) {
  if (!b->data) return;
  const float* bv = (const float*)b->data;
  for (int i = 0; i < b->rows * b->cols; ++i) y[i] += bv[i];
}

/*
 * ForwardToken CPU branch, src/forward.cc:776-807, with ForwardLayer
 * (src/forward.cc:650-707): RMSNorm -> QKV (+bias) -> RoPE -> KV write ->
 * attention -> wo -> residual -> RMSNorm -> gate/up -> SwiGLU -> down ->
 * residual; then final RMSNorm and lm_head (src/forward.cc:762-766).
 */
int mlp_forward_token(mlp_ctx* cx, int token, int pos, float* logits) {
  mlp_model* m = cx->m;
  const mlp_config* c = &m->c;
  if (token < 0 || token >= c->vocab_size)
    return fail(-2, "ForwardToken token id out of range");
  if (pos < 0 || pos >= c->max_seq_len)
    return fail(-2, "ForwardToken position out of range");
  const weight_t* emb = &m->global[MLP_W_TOKEN_EMBEDDING];
  if (!emb->data) return fail(-1, "ForwardToken: missing token_embedding");
  memcpy(cx->x, (const float*)emb->data + (size_t)token * c->dim,
         sizeof(float) * (size_t)c->dim);
  size_t kd = (size_t)c->n_kv_heads * c->head_dim;
  for (int l = 0; l < c->n_layers; ++l) {
    weight_t* L = &m->layer[l * 12];
#define W(kind) (&L[(kind)-3])
    mlp_rmsnorm(cx->x, (const float*)W(MLP_W_ATTENTION_NORM)->data, c->dim,
                c->rms_norm_eps, cx->h);
    int rc = lin(W(MLP_W_WQ), cx->h, cx->q);
    rc |= lin(W(MLP_W_WK), cx->h, cx->k);
    rc |= lin(W(MLP_W_WV), cx->h, cx->v);
    if (rc) return rc;
    add_bias(cx->q, W(MLP_W_BQ));
    add_bias(cx->k, W(MLP_W_BK));
    add_bias(cx->v, W(MLP_W_BV));
    mlp_rope(cx->q, c->n_heads, cx->k, c->n_kv_heads, c->head_dim, pos,
             c->rope_theta, c->rope_type);
    if (cx->kv_bf16)
      for (size_t i = 0; i < kd; ++i) {
        cx->k[i] = bf16_round(cx->k[i]);
        cx->v[i] = bf16_round(cx->v[i]);
      }
    size_t slot_off = ((size_t)l * c->max_seq_len + pos) * kd;
    memcpy(cx->keys + slot_off, cx->k, kd * sizeof(float));
    memcpy(cx->values + slot_off, cx->v, kd * sizeof(float));
    mlp_attention(cx->q, cx->keys, cx->values, l, c->max_seq_len, c->n_heads,
                  c->n_kv_heads, c->head_dim, pos, 0, cx->att);
    if ((rc = lin(W(MLP_W_WO), cx->att, cx->proj))) return rc;
    for (int i = 0; i < c->dim; ++i) cx->x[i] = cx->x[i] + cx->proj[i];
    mlp_rmsnorm(cx->x, (const float*)W(MLP_W_FFN_NORM)->data, c->dim,
                c->rms_norm_eps, cx->h);
    rc = lin(W(MLP_W_GATE), cx->h, cx->gate);
    rc |= lin(W(MLP_W_UP), cx->h, cx->up);
    if (rc) return rc;
    mlp_swiglu(cx->gate, cx->up, c->hidden_dim, cx->act);
    if ((rc = lin(W(MLP_W_DOWN), cx->act, cx->proj))) return rc;
    for (int i = 0; i < c->dim; ++i) cx->x[i] = cx->x[i] + cx->proj[i];
#undef W
  }
  mlp_rmsnorm(cx->x, (const float*)m->global[MLP_W_FINAL_NORM].data, c->dim,
              c->rms_norm_eps, cx->h);
  return lin(&m->global[MLP_W_LM_HEAD], cx->h, logits);
}

/*
 * mlport — CPU restatement of mini-llama's decode forward path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the oracle the CUDA path is checked
 * against. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may load it. The product library never links or calls it.
 *
 * Every function restates the reference's CPU algorithm and cites the
 * reference file:line it follows (paths are relative to the reference
 * project root). Arithmetic is single-precision, sequential, and compiled
 * with -ffp-contract=off, like the reference's default x86-64 build, so the
 * results are bit-identical to the reference CPU path on the same inputs
 * (pinned by tests/test_oracle_port.py against oracle/_ref).
 */
#ifndef MLPORT_H
#define MLPORT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* QuantType order of include/mini_llama/quantized_tensor.h:18-23. */
enum { MLP_F32 = 0, MLP_Q8_0 = 1, MLP_Q4_0 = 2, MLP_Q4_1 = 3 };

/* Weight kinds, in the upload order of src/model.cc:353-369. */
enum {
  MLP_W_TOKEN_EMBEDDING = 0,
  MLP_W_FINAL_NORM = 1,
  MLP_W_LM_HEAD = 2,
  MLP_W_ATTENTION_NORM = 3,
  MLP_W_WQ = 4,
  MLP_W_WK = 5,
  MLP_W_WV = 6,
  MLP_W_BQ = 7,
  MLP_W_BK = 8,
  MLP_W_BV = 9,
  MLP_W_WO = 10,
  MLP_W_FFN_NORM = 11,
  MLP_W_GATE = 12,
  MLP_W_UP = 13,
  MLP_W_DOWN = 14,
  MLP_W_COUNT = 15
};

float mlp_fp16_to_f32(uint16_t h);
uint16_t mlp_f32_to_fp16(float f);
/* Bytes of one 32-element block (34/18/20); 4 for F32 (per element). */
size_t mlp_block_bytes(int qtype);
/* Bytes of a [rows, cols] weight in GGUF layout. */
size_t mlp_weight_bytes(int qtype, int rows, int cols);

int mlp_dequant(int qtype, const void* w, int rows, int cols, float* out);
int mlp_quantize(int qtype, const float* src, int rows, int cols, void* out);
int mlp_linear(int qtype, const float* x, int rows, int in_features,
               const void* w, int out_features, float* y);
void mlp_rmsnorm(const float* x, const float* w, int n, float eps, float* y);
void mlp_rope(float* q, int n_heads, float* k, int n_kv_heads, int head_dim,
              int pos, float theta, int neox);
void mlp_softmax(const float* x, int n, float* y);
void mlp_swiglu(const float* gate, const float* up, int n, float* y);
float mlp_attention_scale(int head_dim);
void mlp_attention(const float* q, const float* keys, const float* values,
                   int layer, int max_seq_len, int n_heads, int n_kv_heads,
                   int head_dim, int pos, int include_current_v, float* out);
int mlp_argmax(const float* x, int n);

typedef struct {
  int vocab_size, dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim,
      max_seq_len;
  float rope_theta, rms_norm_eps;
  int rope_type; /* 0 = normal, 1 = NeoX */
} mlp_config;

typedef struct mlp_model mlp_model;
typedef struct mlp_ctx mlp_ctx;

mlp_model* mlp_model_create(const mlp_config* cfg);
void mlp_model_destroy(mlp_model* m);
/* Copies the weight. rows/cols describe [out, in] (1-D tensors: rows=1). */
int mlp_model_set_weight(mlp_model* m, int kind, int layer, int qtype,
                         int rows, int cols, const void* data, size_t bytes);
mlp_ctx* mlp_ctx_create(mlp_model* m);
void mlp_ctx_destroy(mlp_ctx* c);
/* ForwardToken: writes vocab_size logits. Returns 0 or a negative error. */
int mlp_forward_token(mlp_ctx* c, int token, int pos, float* logits);
/* Not a reference mode: K and V rounded to bf16 (nearest even) when written
 * to the cache, the GPU library's bf16 KV option. */
void mlp_ctx_set_kv_bf16(mlp_ctx* c, int on);
/* The context's fp32 KV cache arrays [L][max_seq][KV][D] (tests fill them). */
void mlp_ctx_kv(mlp_ctx* c, float** keys, float** values);
const char* mlp_last_error(void);

#ifdef __cplusplus
}
#endif

#endif

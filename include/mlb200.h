/*
 * mlb200.h — C ABI of the B200 (sm_100a) decode forward path.
 *
 * This is the drop-in boundary under mini-llama's device branch. Each entry
 * point names the reference interface it replaces (file:line in the
 * reference project). All functions return MLB_OK (0) or a negative status;
 * mlb_last_error() gives the message for the calling thread. MLB_ERR_RANGE
 * corresponds to the reference's std::out_of_range (bad token, position,
 * layer or head index) and MLB_ERR_INVALID to its std::runtime_error, so a C++
 * shim can rethrow with the same exception types and messages.
 *
 * Pointers named *_dev are device pointers on `device_id`; `stream` is a
 * cudaStream_t (NULL means the legacy default stream). No signature carries a
 * framework type. Weights use the GGUF block layouts of the reference
 * (include/mini_llama/quantized_tensor.h:26-44): Q8_0 = {fp16 d; int8 qs[32]}
 * (34 B), Q4_0 = {fp16 d; uint8 qs[16]} (18 B), Q4_1 = {fp16 d; fp16 m; uint8
 * qs[16]} (20 B), row-major [out_features, in_features] with each row padded
 * to whole 32-element blocks; F32 weights are plain row-major floats.
 */
#ifndef MLB200_H
#define MLB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLB_OK 0
#define MLB_ERR_INVALID (-1)  /* reference: std::runtime_error */
#define MLB_ERR_RANGE (-2)    /* reference: std::out_of_range */
#define MLB_ERR_CUDA (-3)     /* a CUDA runtime call failed */
#define MLB_ERR_NCCL (-4)     /* an NCCL call failed */
#define MLB_ERR_TIMEOUT (-5)  /* a bounded device wait gave up */

/* QuantType order of include/mini_llama/quantized_tensor.h:18-23. */
#define MLB_F32 0
#define MLB_Q8_0 1
#define MLB_Q4_0 2
#define MLB_Q4_1 3

/* RopeType, include/mini_llama/model.h:11-14. */
#define MLB_ROPE_NORMAL 0
#define MLB_ROPE_NEOX 1

/* Weight kinds in the upload order of UploadModelWeightsToCuda,
 * src/model.cc:353-369. */
#define MLB_W_TOKEN_EMBEDDING 0
#define MLB_W_FINAL_NORM 1
#define MLB_W_LM_HEAD 2
#define MLB_W_ATTENTION_NORM 3
#define MLB_W_WQ 4
#define MLB_W_WK 5
#define MLB_W_WV 6
#define MLB_W_BQ 7
#define MLB_W_BK 8
#define MLB_W_BV 9
#define MLB_W_WO 10
#define MLB_W_FFN_NORM 11
#define MLB_W_GATE 12
#define MLB_W_UP 13
#define MLB_W_DOWN 14

/* Attention modes of a decode context. CPU_COMPAT reproduces the reference
 * CPU path, whose V sum stops before the current position while the softmax
 * covers it (src/forward.cc:501-518); STANDARD sums V over t <= pos like the
 * reference GPU kernel (src/cuda_attention.cu:192-203). */
#define MLB_ATTN_CPU_COMPAT 0
#define MLB_ATTN_STANDARD 1

/* KV cache element types of a batch (mlb_batch_create_kv). F32 is the
 * reference's CudaKvCache layout and the parity mode; BF16 stores each K and
 * V value rounded to bf16 (nearest even) and halves the cache's bytes. */
#define MLB_KV_F32 0
#define MLB_KV_BF16 1

/* Thread-local message of the last failed call on this thread. */
const char* mlb_last_error(void);

/* Replaces CudaQuantBuilt/CudaOpsBuilt/CudaAttentionBuilt/CudaRuntimeBuilt
 * (include/mini_llama/cuda_quant.h:10, cuda_ops.h:9, cuda_attention.h:9,
 * cuda_runtime.h:26): 1 when the sm_100a kernels are compiled in. */
int mlb_built(void);

/* Replaces CudaDeviceCount (include/mini_llama/cuda_runtime.h:27). */
int mlb_device_count(int* count);

/* Failure-detection self-test; no counterpart in the reference (whose device
 * code has no waits). Every wait inside the decode-step kernel is bounded: it
 * gives up after a limit, records MLB_ERR_TIMEOUT and the wait site in the
 * context's status word, and returns, so a stuck peer or a lost copy becomes
 * an error status instead of a hung GPU. This runs one of those waits on
 * `device` against something that never comes, with a limit of `limit_ms`
 * (0 < limit_ms <= 1000): which = 0 waits on a shared-memory ring slot whose
 * copy never lands (the weight stream's mbarrier wait), which = 1 on a grid
 * barrier that no other CTA joins. Writes the recorded status code
 * (MLB_ERR_TIMEOUT when the wait gave up) and site (900 + which); the
 * device stays usable. Synchronous. */
int mlb_wait_selftest(int device, int which, double limit_ms, int* code, int* where);

/* ------------------------------------------------------------------ linear
 * y[rows, out] = x[rows, in] * W^T over raw GGUF blocks on the device.
 * Replaces CudaQ80LinearDeviceInput / CudaQ40LinearDeviceInput /
 * CudaQ41LinearDeviceInput (include/mini_llama/cuda_quant.h:18,24,30) and,
 * for qtype MLB_F32, CudaLinearDeviceInput (include/mini_llama/cuda_matmul.h:18).
 * block_count must equal out * ceil(in / 32) (F32: out * in), the check of
 * src/cuda_quant.cu:206-223. */
int mlb_linear(int qtype, const float* x_dev, int rows, int in_features,
               const void* w_dev, size_t block_count, int out_features,
               float* y_dev, int device_id, void* stream);

/* Host activations and host weights, optional host bias (may be NULL):
 * replaces CudaQ80Linear / CudaQ40Linear / CudaQ41Linear
 * (include/mini_llama/cuda_quant.h:12,20,26) and CudaLinear
 * (include/mini_llama/cuda_matmul.h:14). Synchronous. */
int mlb_linear_host(int qtype, const float* x, int rows, int in_features,
                    const void* w, size_t block_count, int out_features,
                    const float* bias, float* y, int device_id);

/* Host activations, device weights, optional host bias: replaces
 * CudaQ80LinearDeviceWeight / CudaQ40LinearDeviceWeight /
 * CudaQ41LinearDeviceWeight (include/mini_llama/cuda_quant.h:14,22,28) and
 * CudaLinearDeviceWeight (include/mini_llama/cuda_matmul.h:16). Synchronous. */
int mlb_linear_device_weight(int qtype, const float* x, int rows,
                             int in_features, const void* w_dev,
                             size_t block_count, int out_features,
                             const float* bias, float* y, int device_id);

/* -------------------------------------------------------- elementwise ops
 * Replace the device-input ops of include/mini_llama/cuda_ops.h:21-37. */
/* CudaRmsNormDeviceWeight (cuda_ops.h:27): y = x / sqrt(mean(x^2)+eps) * w. */
int mlb_rmsnorm(const float* x_dev, const float* w_dev, int n, float eps,
                float* y_dev, int device_id, void* stream);
/* CudaSiluDeviceInput (cuda_ops.h:29). */
int mlb_silu(const float* x_dev, int n, float* y_dev, int device_id, void* stream);
/* CudaElementwiseMulDeviceInput (cuda_ops.h:31). */
int mlb_mul(const float* a_dev, const float* b_dev, int n, float* y_dev,
            int device_id, void* stream);
/* CudaElementwiseAddDeviceInput / DeviceWeight (cuda_ops.h:33,35). */
int mlb_add(const float* a_dev, const float* b_dev, int n, float* y_dev,
            int device_id, void* stream);
/* CudaSoftmax (cuda_ops.h:19), on device data. */
int mlb_softmax(const float* x_dev, int n, float* y_dev, int device_id, void* stream);
/* CudaEmbeddingLookupDeviceWeight (cuda_ops.h:23): y = table[token, :]. */
int mlb_embedding(const float* table_dev, int vocab, int dim, int token,
                  float* y_dev, int device_id, void* stream);
/* CudaRopeDeviceInput (cuda_ops.h:37): in-place RoPE of q [n_heads, D] and
 * k [n_kv_heads, D]; the angles are evaluated on the host exactly as the
 * reference CPU path does (src/ops.cc:143-178). */
int mlb_rope(float* q_dev, float* k_dev, int n_heads, int n_kv_heads,
             int head_dim, int pos, float theta, int rope_type, int device_id,
             void* stream);
/* Index of the largest logit, lowest index on ties (ArgMax, src/ops.cc:220). */
int mlb_argmax(const float* x_dev, int n, int* index_host, int device_id, void* stream);

/* ------------------------------------------------------ KV cache + attention
 * The cache is two fp32 arrays [n_layers][max_seq_len][n_kv_heads][head_dim]
 * (keys, values), the layout of CudaKvCache (src/cuda_kv_cache.cc:328-333). */
/* CudaKvCache::WriteDevice (include/mini_llama/cuda_kv_cache.h:28). */
int mlb_kv_write(float* keys_dev, float* values_dev, int n_layers,
                 int max_seq_len, int n_kv_heads, int head_dim, int layer,
                 int pos, const float* k_dev, const float* v_dev, int device_id,
                 void* stream);
/* CudaAttentionDecodeDeviceInput (include/mini_llama/cuda_attention.h:13):
 * out[n_heads, D] = softmax(q K^T / sqrt(D)) V over positions [0, pos] of
 * `layer`, GQA head map h / (n_heads / n_kv_heads). mode is MLB_ATTN_*. */
int mlb_attention_decode(const float* q_dev, const float* keys_dev,
                         const float* values_dev, int n_layers, int max_seq_len,
                         int layer, int pos, int n_heads, int n_kv_heads,
                         int head_dim, int mode, float* out_dev, int device_id,
                         void* stream);

/* The same attention as mlb_attention_decode, for callers that must not
 * allocate device memory during the call: hosts whose device memory is owned by
 * their own allocator under a fixed budget, and latency-sensitive decode loops
 * that cannot afford cudaMalloc/cudaFree (cudaFree synchronises the device).
 * It has no counterpart in the reference (whose attention allocates its score
 * buffer per call, src/cuda_attention.cu:268-273). Its split-K scratch is a
 * fixed array inside the library: 4 MiB of partials (at most 2^20 floats for
 * one split: n_kv_heads * (n_heads / n_kv_heads) * (head_dim + 2)) plus
 * counters for at most 1024 KV heads; larger shapes are rejected with
 * MLB_ERR_INVALID. Every GPU that loads the library holds this array until the
 * process exits. The first call on a device looks up the array's device
 * address, so make that first call before any stream capture. All calls share
 * the array: calls that overlap on the GPU (other streams, other threads) race
 * and give wrong results; run them one after another. Asynchronous on `stream`
 * (no host synchronisation, unlike mlb_attention_decode): synchronise `stream`
 * before reading out_dev. The looked-up address is kept for the life of the
 * process; it does not survive cudaDeviceReset (which reloads the module), so
 * do not call this after resetting a device it has run on. */
int mlb_attention_decode_noalloc(const float* q_dev, const float* keys_dev,
                                 const float* values_dev, int n_layers,
                                 int max_seq_len, int layer, int pos, int n_heads,
                                 int n_kv_heads, int head_dim, int mode,
                                 float* out_dev, int device_id, void* stream);

/* --------------------------------------------------------- prepared weights
 * A weight repacked once into the B200 GEMV layout (what the decode path
 * streams). No reference counterpart as an API: it is the device-resident
 * form UploadModelWeightsToCuda keeps (src/model.cc:345-374). */
typedef struct mlb_qmatrix mlb_qmatrix;
int mlb_qmatrix_create(int qtype, const void* w, int w_is_host,
                       int out_features, int in_features, int device_id,
                       mlb_qmatrix** out);
/* Fills a prepared weight with the seeded synthetic generator (GGUF blocks of
 * N(0,1) * scale quantised like the reference, or raw random blocks when
 * raw != 0); bit-identical to the host generator. */
int mlb_qmatrix_synthesize(int qtype, int out_features, int in_features,
                           uint64_t seed, uint64_t stream_id, int raw,
                           int device_id, mlb_qmatrix** out);
/* y[rows, out] = x[rows, in] * W^T, device pointers, on `stream`. Up to 4
 * rows run the batch-1 GEMV (mma.sync over in-register dequantised codes);
 * more rows run mlb_qmatrix_gemm. */
int mlb_qmatrix_gemv(mlb_qmatrix* m, const float* x_dev, int rows, float* y_dev,
                     void* stream);
/* The same product on the tcgen05 tensor cores for any row count (64 rows per
 * pass of the weights): codes dequantised to exact fp16 hi + lo pairs in
 * tensor memory, activations as fp16 hi + lo, fp32 accumulation. Replaces the
 * per-row loop a batch takes through LinearQ80/Q40/Q41 (src/quant.cc:365-471;
 * ForwardBatch, src/batch.cc:35-50, runs one token at a time). Quantised types
 * only. Its scratch is allocated with the matrix, so calls can be captured in a
 * CUDA graph. */
int mlb_qmatrix_gemm(mlb_qmatrix* m, const float* x_dev, int rows, float* y_dev,
                     void* stream);
/* The prepared weight dequantised back to fp32, out_dev[out_features *
 * in_features] row-major, decoded from the repacked layout the GEMV streams.
 * Replaces DequantizeFromQ80 / DequantizeFromQ40 / DequantizeFromQ41
 * (include/mini_llama/quant.h; src/quant.cc:170-361) and gives the same bits:
 * Q4_0 (q - 8) * d, Q4_1 q * d + m, Q8_0 d * q in fp32. Quantised types only.
 * Asynchronous on `stream`. */
int mlb_qmatrix_dequant(const mlb_qmatrix* m, float* out_dev, void* stream);
/* Algorithmic GGUF bytes of the weight (what a GEMV must stream). */
size_t mlb_qmatrix_bytes(const mlb_qmatrix* m);
int mlb_qmatrix_destroy(mlb_qmatrix* m);

/* ---------------------------------------------------- model and decode step
 * mlb_config mirrors ModelConfig (include/mini_llama/model.h:21-33). */
typedef struct {
  int vocab_size, dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim,
      max_seq_len;
  float rope_theta, rms_norm_eps;
  int rope_type;
} mlb_config;

typedef struct mlb_model mlb_model;
typedef struct mlb_context mlb_context;

/* The shard one tensor-parallel rank keeps. wq/bq rows and wo input columns:
 * query heads [q_head0, q_head0 + q_heads) (times head_dim); wk/wv/bk/bv rows:
 * KV heads [kv_head0, ...); w_gate/w_up rows and w_down input columns: FFN
 * hidden rows [ffn_row0, ffn_row0 + ffn_rows), whole 32-row blocks split as
 * evenly as the blocks allow; lm_head rows: vocabulary [vocab_row0, ...).
 * Embedding and norms are replicated. */
typedef struct {
  int q_head0, q_heads;
  int kv_head0, kv_heads;
  int ffn_row0, ffn_rows;
  int vocab_row0, vocab_rows;
} mlb_tp_shard;

/* Computes the shard of rank tp_rank of tp_size on the host (no device, no
 * communicator). Returns MLB_ERR_INVALID, with the reason in mlb_last_error(),
 * when the config cannot be split over tp_size ranks. No reference
 * counterpart (the reference runs on one device); mlb_model_create uses it. */
int mlb_tp_plan(const mlb_config* cfg, int tp_rank, int tp_size, mlb_tp_shard* out);

/* Replaces UploadModelWeightsToCuda (include/mini_llama/model.h:103) together
 * with mlb_model_set_weight / mlb_model_finalize. With tp_size > 1 the model
 * holds this rank's tensor-parallel shard (wq/wk/wv/w_gate/w_up split by
 * output rows, wo/w_down by input columns, lm_head by vocabulary rows) and
 * joins an NCCL communicator built from nccl_id (128 bytes from
 * mlb_nccl_unique_id on rank 0); tp_size == 1 ignores nccl_id. */
int mlb_model_create(const mlb_config* cfg, int device_id, int tp_rank,
                     int tp_size, const void* nccl_id, mlb_model** out);
/* Uploads one weight given in full (unsharded) reference layout from host
 * memory; the model keeps only its shard, repacked. kind is MLB_W_*, layer is
 * ignored for the three global tensors. 1-D tensors use rows = 1. */
int mlb_model_set_weight(mlb_model* m, int kind, int layer, int qtype, int rows,
                         int cols, const void* host_data, size_t bytes);
/* Generates every weight on the device with the seeded synthetic generator:
 * linear weights N(0,0.02) quantised to qtype, norms 1.0, embedding
 * N(0,0.02) fp32, and q/k/v biases N(0,0.02) when with_bias != 0. */
int mlb_model_synthesize(mlb_model* m, int qtype, uint64_t seed, int with_bias);
/* Checks that every weight is present and builds the decode plan. */
int mlb_model_finalize(mlb_model* m);
/* The ModelConfig that LoadGgufModel builds from a GGUF v3 file's metadata
 * (BuildConfig, src/gguf_loader.cc:13-88: qwen2.* keys, else llama.* keys,
 * else 0; NeoX RoPE for general.architecture "qwen2"; vocab_size = length of
 * tokenizer.ggml.tokens; head_dim = dim / n_heads). Host only (no device).
 * Parse and config errors return MLB_ERR_INVALID with the reference's
 * messages ("GGUF parse error: invalid GGUF magic", "... unsupported GGUF
 * version: 2", "Failed to build config: ..."). */
int mlb_gguf_read_config(const char* path, mlb_config* out);
/* Replaces LoadGgufModel (src/gguf_loader.cc:302-418) followed by
 * UploadModelWeightsToCuda (src/model.cc:345-374): parses the GGUF v3 file,
 * creates the model (tensor-parallel shard as mlb_model_create), uploads the
 * tensors the model uses straight from the memory-mapped file through pinned
 * staging buffers (this rank's rows only) and finalizes. Tensor names and
 * shapes follow MapTensorName / MapShape; a missing output.weight ties the
 * lm_head to the embedding; quantised or F16 norms, biases and embeddings are
 * widened to F32 with the reference's dequantisation. Unlike the reference,
 * F16 linear weights are accepted (widened to F32, exact); quantised rows must
 * be whole 32-element blocks. max_seq_len > 0 replaces the file's
 * context_length (the KV cache size); bytes_uploaded (optional) receives the
 * bytes copied to the device. */
int mlb_model_load_gguf(const char* path, int device_id, int tp_rank, int tp_size,
                        const void* nccl_id, int max_seq_len, mlb_model** out,
                        size_t* bytes_uploaded);
int mlb_model_destroy(mlb_model* m);
/* Resident bytes of the weights on this device (ModelCudaMemoryBytes,
 * include/mini_llama/model.h:119) and algorithmic GGUF bytes one decode step
 * streams from HBM on this rank. */
int mlb_model_bytes(const mlb_model* m, size_t* resident, size_t* per_step_weights);

/* Replaces MiniLlamaContext's CUDA KV cache (include/mini_llama/context.h:13,
 * CudaKvCache::Reset src/cuda_kv_cache.cc:60-92): allocates and zeroes the
 * fp32 KV cache for max_seq_len positions and all decode buffers once. */
int mlb_context_create(mlb_model* m, int attention_mode, mlb_context** out);
/* The same with the KV cache element type (MLB_KV_F32 or MLB_KV_BF16; the
 * reference's CudaKvCache is fp32 only). A bf16 cache runs on the decode step
 * kernel only (models the step kernel cannot take are refused, and
 * mlb_context_set_step_kernel(c, 0) fails); its results follow the reference
 * CPU path with every K and V value rounded to bf16 when written. */
int mlb_context_create_kv(mlb_model* m, int attention_mode, int kv_type, mlb_context** out);
int mlb_context_destroy(mlb_context* c);
/* Clears the KV cache (CudaKvCache::Clear, src/cuda_kv_cache.cc:96-110). */
int mlb_context_reset(mlb_context* c);
/* Fills positions [0, n_pos) of every layer's K and V cache rows (this rank's
 * KV heads) with seeded values: element (pos, kv_head, d) of layer l is the
 * generator's N(0,1) draw at index (pos * n_kv_heads + kv_head) * head_dim + d
 * of stream 15 * 2^20 + l (K) or 16 * 2^20 + l (V), times scale. A decode
 * state at depth n_pos for benchmarks and tests without n_pos decode steps.
 * No reference counterpart (the reference fills its cache only by decoding).
 * Synchronous. */
int mlb_context_fill_kv(mlb_context* c, int n_pos, uint64_t seed, float scale);

/* Replaces ForwardToken's device branch (src/forward.cc:776-794): runs one
 * decode step for `token` at `pos` and copies the vocab_size logits to host
 * memory. Validation follows ValidateForwardInputs (src/forward.cc:53-79). */
int mlb_forward_token(mlb_context* c, int token, int pos, float* logits_host);
/* Same step with the logits left on the device; returns the device pointer
 * in *logits_dev (valid until the next step). Asynchronous on the context's
 * stream; mlb_context_sync waits for it. */
int mlb_forward_token_device(mlb_context* c, int token, int pos,
                             const float** logits_dev);
int mlb_context_sync(mlb_context* c);
/* Greedy decode kept on the device: step 0 feeds `token` at `pos`, each later
 * step feeds the previous step's argmax (ArgMax tie rule). Writes n_steps
 * token ids (the argmax of each step) to tokens_host. One CUDA graph launch
 * per step, no host round trip between steps. */
int mlb_decode_greedy(mlb_context* c, int token, int pos, int n_steps,
                      int* tokens_host);

/* -------------------------------------------------------------- sampling
 * A sampler is MiniSampler (include/mini_llama/sampler.h): a std::mt19937
 * seeded with `seed` (0 = a random seed, as the reference), its state
 * resident on device_id. mlb_sample is MiniSampler::Sample
 * (src/sampler.cc:172-183) over n logits in device memory: temperature <
 * 1e-6 or top_k == 1 is greedy (first index of the maximum, no draw); top_k
 * > 1 samples among the top_k largest logits (ties: lower index first);
 * top_k == 0 among all. The generator's draws equal the reference's word for
 * word; the softmax sums run on the device in a fixed order, so a sample
 * differs from the reference's only when the uniform draw falls within
 * rounding distance of a candidate boundary. Errors, with the reference's
 * messages: empty logits, negative top_k, negative or non-finite temperature
 * (before any device work), non-finite logits (after the sample, MLB_ERR_INVALID).
 * top_k above 4096 (after clamping to n) is rejected: the device sorts at
 * most 4096 candidates. mlb_sample syncs the sampler's own stream. */
typedef struct mlb_sampler mlb_sampler;
int mlb_sampler_create(int device_id, unsigned int seed, mlb_sampler** out);
int mlb_sampler_destroy(mlb_sampler* s);
int mlb_sample(mlb_sampler* s, const float* logits_dev, int n, float temperature, int top_k,
               int* out_id);
/* mlb_decode_greedy with the sampler's choice in place of the argmax at every
 * step (RunGenerate's decode loop, src/main.cc:883-912, without the per-step logits
 * download): one full-logits step and one sampling kernel per step, on the
 * context's stream, with no host round trip between steps. Tensor-parallel
 * ranks each pass a sampler seeded alike: every rank holds the whole logits
 * row, so all draw and pick the same ids. The sampler must be on the
 * context's device. */
int mlb_decode_sample(mlb_context* c, mlb_sampler* s, float temperature, int top_k, int token,
                      int pos, int n_steps, int* tokens_host);
/* The context's stream (cudaStream_t), for timing with events. */
void* mlb_context_stream(mlb_context* c);
/* Number of kernels one decode step launches on this rank. */
int mlb_context_kernels_per_step(const mlb_context* c);
/* Selects how a single-GPU decode step runs: 1 = the persistent step kernel
 * (one cooperative launch computes the whole step; the default wherever the
 * model allows it), 0 = one kernel per op in a CUDA graph. Asking for 1 on a
 * model the step kernel does not take (F32 or mixed quant types, head_dim >
 * 128 or not a multiple of 4, very large GQA groups, tensor parallel with dim
 * above 8192)
 * returns MLB_ERR_INVALID and mlb_last_error() gives the reason. No reference
 * counterpart: the reference always launches one kernel per op
 * (src/forward.cc:700-794). */
int mlb_context_set_step_kernel(mlb_context* c, int enable);
/* 1 when this context's steps run as the persistent step kernel, else 0. */
int mlb_context_step_kernel(const mlb_context* c);

/* Phase trace of the step kernel (a diagnostic; no reference counterpart).
 * enable = 1 makes every later step record, per phase and CTA, two global-
 * timer stamps (ns): the start of the phase's work after the grid barrier
 * ahead of it, and its end before the next one; the context must be on the
 * step kernel. mlb_context_step_trace_read sets *nphases and *grid; when
 * stamps is non-null and cap >= nphases * grid * 2 it syncs the context's
 * stream, copies the stamps of the last traced step there ([phase][cta][2])
 * and clears the record (a read with no whole traced step since the last one
 * fails); otherwise it only reports the sizes. Phases in order: per layer
 * QKV projection, attention, wo, gate/up, w_down; then lm_head. */
int mlb_context_step_trace(mlb_context* c, int enable);
int mlb_context_step_trace_read(mlb_context* c, uint64_t* stamps, size_t cap, int* nphases,
                                int* grid);

/* ------------------------------------------------------------------ batches
 * Rows of (token, position) go through every layer together: the weights
 * stream once per pass of up to 64 rows through the tcgen05 tensor-core GEMM
 * (mlb_qmatrix_gemm) with the fused prologue/epilogues of the single-token
 * step, and attention runs one CTA per (KV head, split, row). Tensor-parallel
 * models all-reduce the wo and w_down partial sums with NCCL. */

/* ForwardBatch (src/batch.cc:35-50) on one context: n_tokens tokens at their
 * positions (strictly increasing: the reference feeds them one ForwardToken
 * at a time, so each token sees the K/V of the ones before it), the KV cache
 * written for every position, the logits of the last token to host. Prompt
 * prefill in passes of 64 rows. Synchronous. */
int mlb_forward_batch(mlb_context* c, int n_tokens, const int* tokens,
                      const int* positions, float* logits_host);

/* A batch of 1..64 independent sequences decoded together, each with its own
 * fp32 KV cache laid out as CudaKvCache's [L][max_seq][KV][D]. The reference
 * has no multi-sequence decode (one MiniLlamaContext per sequence); a batch
 * replaces that many contexts stepping in lockstep. */
typedef struct mlb_batch mlb_batch;
int mlb_batch_create(mlb_model* m, int n_seqs, int attention_mode, mlb_batch** out);
/* The same with the KV cache element type (MLB_KV_F32 or MLB_KV_BF16;
 * cuda_kv_cache.cc:60-92 keeps fp32 only). A bf16 cache needs head_dim a
 * multiple of 4 up to 128 and 1, 2, 4 or 8 query heads per KV head; its
 * results follow the reference CPU path with every K and V value rounded to
 * bf16 when written, not the fp32 path. */
int mlb_batch_create_kv(mlb_model* m, int n_seqs, int attention_mode, int kv_type,
                        mlb_batch** out);
int mlb_batch_destroy(mlb_batch* b);
/* Clears every sequence's KV cache. */
int mlb_batch_reset(mlb_batch* b);
/* mlb_context_fill_kv for sequence `seq` (the same seeded values). */
int mlb_batch_fill_kv(mlb_batch* b, int seq, int n_pos, uint64_t seed, float scale);
/* One pass of n_rows rows (seq_ids[i], tokens[i], positions[i]); rows of one
 * sequence need strictly increasing positions. Writes each row's greedy
 * token (ArgMax tie rule) to next_tokens_host[i] and, when logits_host is not
 * NULL, its logits to logits_host[i * vocab]. Synchronous. */
int mlb_batch_forward(mlb_batch* b, int n_rows, const int* seq_ids, const int* tokens,
                      const int* positions, float* logits_host, int* next_tokens_host);
/* Greedy decode of all n_seqs sequences in lockstep for n_steps steps:
 * sequence s starts from tokens[s] at positions[s]; tokens_out[step * n_seqs
 * + s] receives the argmax of each step. One CUDA graph launch per step, no
 * host round trip between steps. */
int mlb_batch_decode_greedy(mlb_batch* b, const int* tokens, const int* positions, int n_steps,
                            int* tokens_out);
/* The batch's stream (cudaStream_t) and the kernels one decode step launches. */
void* mlb_batch_stream(mlb_batch* b);
int mlb_batch_kernels_per_step(const mlb_batch* b);

/* 128-byte NCCL unique id for building a tensor-parallel communicator. */
int mlb_nccl_unique_id(void* out128);

#ifdef __cplusplus
}
#endif

#endif

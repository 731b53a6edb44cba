// runtime.cuh — model, context and decode step (host side).
#pragma once

#include <nccl.h>

#include <map>
#include <memory>
#include <vector>

#include "attention.cuh"
#include "gemv.cuh"
#include "step.cuh"

namespace mlb {

// Device allocation that frees itself.
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  explicit DevBuf(size_t n) { alloc(n); }
  void alloc(size_t n);
  void reset();
  ~DevBuf() { reset(); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) { reset(); p = o.p; bytes = o.bytes; o.p = nullptr; o.bytes = 0; }
    return *this;
  }
  template <class T> T* as() const { return static_cast<T*>(p); }
};

struct RawTensor {  // one uploaded GGUF tensor shard on the device, before fusing
  int qtype = 0, rows = 0, cols = 0;  // shard shape
  size_t pitch = 0;
  DevBuf buf;
};

struct LayerPlan {
  DevBuf attn_norm, ffn_norm, bias;  // bias: fused local [q | k | v] or empty
  QMatrix qkv, wo, gateup, down;
  DevBuf qkv_buf, wo_buf, gateup_buf, down_buf;
  int qkv_k_off = 0, qkv_v_off = 0;
};

struct ModelImpl {
  mlb_config cfg{};
  int device = 0;
  int tp_rank = 0, tp_size = 1;
  ncclComm_t comm = nullptr;
  // this rank's shard
  int q_heads = 0, kv_heads = 0, q_head0 = 0, kv_head0 = 0;
  int ffn_rows = 0, ffn_row0 = 0;     // hidden rows (block aligned)
  int vocab_rows = 0, vocab_row0 = 0, vocab_pad = 0;
  bool neox = false;
  bool finalized = false;
  // weights
  DevBuf embedding, final_norm;
  QMatrix lm_head;
  DevBuf lm_head_buf;
  std::vector<LayerPlan> layers;
  DevBuf rope;  // [max_seq][D/2] float2
  // pending uploads (kind, layer) -> shard on device
  std::map<std::pair<int, int>, RawTensor> pending;
  cudaStream_t stream = nullptr;
  size_t resident_bytes() const;
  size_t step_weight_bytes() const;
};

// Where an upload of weight (kind, layer) lands on this rank: the full
// tensor's shape, whether it must be F32, and the shard kept: rows
// [first, first + count) of the tensor, or for the q/k/v biases (by_cols)
// columns [first, first + count) of its single row.
struct WeightSlot {
  int rows = 0, cols = 0;
  bool f32_only = false, by_cols = false;
  int first = 0, count = 0;
  std::string name;
};
WeightSlot model_weight_slot(const ModelImpl& m, int kind, int layer);
// Hands a shard already on the device to the model (finalize fuses it).
void model_put_raw(ModelImpl& m, int kind, int layer, RawTensor&& t);

// GGUF files (gguf.cu): a parsed, memory-mapped file; its model config
// (BuildConfig semantics); the upload of every tensor the model uses (this
// rank's shards) through pinned staging buffers, returning the bytes copied.
struct GgufFile;
GgufFile* gguf_open(const char* path);
void gguf_close(GgufFile* g);
mlb_config gguf_config(const GgufFile& g);
size_t gguf_upload(ModelImpl& m, const GgufFile& g);

struct BatchEngine;  // batch.cu: scratch of one batched pass
void batch_engine_free(BatchEngine* e);

struct ContextImpl {
  // ForwardBatch on this context (prompt prefill through the tensor-core
  // GEMM), created on first use
  BatchEngine* batch = nullptr;
  ModelImpl* m = nullptr;
  int attention_mode = MLB_ATTN_CPU_COMPAT;
  cudaStream_t stream = nullptr;
  DevBuf keys, values;        // [L][S][KV_local][D], fp32 or (kv_bf16) bf16 elements
  bool kv_bf16 = false;
  // layer l's base of the keys / values, typed as the kernels take it
  float* kv_layer(const DevBuf& b, int l) const;
  DevBuf xa, xb, y, q, attn, hidden, logits_local, logits;
  DevBuf ss_x;  // step kernel: per-tile sums of squares of xa, then of xb
  DevBuf gemv_ws, gemv_cnt, attn_ws, attn_cnt, status;
  DevBuf scalars;             // int: token, pos, step, next token ; then tokens[max_seq]
  DevBuf argmax_key;          // u64 packed (logit, index) of the step's greedy argmax
  int* h_scalars = nullptr;   // pinned: token, pos
  float* h_logits = nullptr;  // pinned
  int* h_tokens = nullptr;    // pinned
  int attn_splits = 1;
  GemvWorkspace ws;
  cudaGraph_t graph = nullptr, graph_greedy = nullptr;
  cudaGraphExec_t exec = nullptr;         // step that also leaves full logits on the device
  cudaGraphExec_t exec_greedy = nullptr;  // step that only produces the next token
  int kernels_per_step = 0;
  // Persistent decode-step kernel (single GPU): plan, phase table, grid sync
  // words and attention workspace. use_step selects it over the per-op graph.
  StepPlan step;
  DevBuf step_phases, step_cta, step_sync, step_attn_ws, step_attn_cnt;
  DevBuf step_trace;      // [nphases][grid][2] u64 (StepArgs::trace) while tracing
  bool trace_on = false;
  // tensor-parallel step kernel: this rank's exchange buffer, the other
  // ranks' buffers mapped here, the exchange descriptor and step counter
  DevBuf xchg, tp_desc, tp_gen;
  TpXchg tpx{};
  std::vector<void*> tp_opened;  // peer mappings to close
  void setup_tp_exchange();
  const float* logits_dev() const;  // where a step leaves the full logits
  bool use_step = false;
  bool direct_launch = false;  // step kernel launched without a graph
  void plan_step();
  void build_graph();
  void record_step(cudaStream_t s, bool pdl, bool full_logits);
  void launch_step(cudaStream_t s);
  void release_graphs();
  void replay(bool greedy);  // one step from the graph (or a direct launch)
  void set_use_step(bool on);
  void set_step_trace(bool on);
  void read_step_trace(unsigned long long* stamps, size_t cap, int* nphases, int* grid);
  void check_status();
  ~ContextImpl();
};

}  // namespace mlb

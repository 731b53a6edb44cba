// batch.cu — batched decode and prompt prefill on the tensor-core GEMM.
//
// Reference: ForwardBatch (src/batch.cc:35-50) runs the tokens of a batch
// one ForwardToken at a time, and the reference has no way to decode several
// sequences together (its KV cache belongs to one MiniLlamaContext). Here one
// pass takes up to 64 rows, each a (sequence, token, position), through every
// layer at once:
//   embedding rows -> per layer:
//     stage x (RMSNorm)   -> QKV GEMM   (epilogue: bias, RoPE at each row's
//                                        position, q rows, K/V into each
//                                        row's sequence cache)
//     attention, one CTA per (KV head, split, row) over each row's positions
//     stage attention     -> wo GEMM    (epilogue: + residual)
//     stage x' (RMSNorm)  -> gate/up    (epilogue: SiLU(gate) * up)
//     stage hidden        -> down GEMM  (epilogue: + residual)
//   stage x (final norm) -> lm_head GEMM (epilogue: logits, greedy argmax per
//                                         row)
// so the weights stream once per pass for all rows. Rows of one sequence
// (prompt prefill) must come with strictly increasing positions: every row's
// K/V is written before attention runs, and row i attends positions <= its
// own, exactly the rows the sequential loop has written by then.
// Under tensor parallelism wo and down store partial sums that an NCCL
// all-reduce adds before the residual, and the per-row greedy keys are
// reduced with max across the vocabulary shards.
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "attention.cuh"
#include "ops.cuh"
#include "qgemm.cuh"
#include "runtime.cuh"

namespace mlb {

namespace {

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) fail(MLB_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

// x[r][:] = table[tok[r]][:]
__global__ void gather_rows_kernel(float* x, const float* table, const int* tok, int rows, int dim) {
  const int r = blockIdx.y;
  if (r >= rows) return;
  const float* src = table + (size_t)tok[r] * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    x[(size_t)r * dim + i] = __ldg(src + i);
}

// End of a decode step for every row: the greedy token (ArgMax tie rule)
// becomes the row's next input, is recorded as out[step][r], the position
// advances and the key is cleared.
__global__ void batch_finalize_kernel(unsigned long long* keys, int* tok, int* pos, int rows,
                                      int* out, int* step) {
  const int r = threadIdx.x;
  const int s = *step;
  __syncthreads();
  if (r < rows) {
    const int t = argmax_index_of(keys[r]);
    tok[r] = t;
    out[(size_t)s * rows + r] = t;
    pos[r] += 1;
    keys[r] = 0ull;
  }
  __syncthreads();
  if (r == 0) *step = s + 1;
}

}  // namespace

// Scratch of one pass of up to max_rows rows (kTcMaxMp at most).
struct BatchEngine {
  ModelImpl* m = nullptr;
  int max_rows = 0;
  int mode = MLB_ATTN_CPU_COMPAT;
  DevBuf x, x2, q, attn, hidden, tmp, logits, staged;
  DevBuf tc_parts, tc_cnt, status;
  TcWorkspace tcws;
  DevBuf attn_ws, attn_cnt;
  int attn_nsplit = 1;
  DevBuf rows_dev;  // int [3][max_rows]: tokens, positions, sequences
  DevBuf keys_dev;  // u64 greedy keys [max_rows]
  DevBuf step_dev;  // int: decode-loop step counter

  int* tok() const { return rows_dev.as<int>(); }
  int* pos() const { return rows_dev.as<int>() + max_rows; }
  int* seq() const { return rows_dev.as<int>() + 2 * max_rows; }

  void init(ModelImpl* model, int rows, int attention_mode) {
    m = model;
    max_rows = rows;
    mode = attention_mode;
    const mlb_config& c = m->cfg;
    const int D = c.head_dim;
    x.alloc((size_t)rows * c.dim * 4);
    x2.alloc((size_t)rows * c.dim * 4);
    tmp.alloc((size_t)rows * c.dim * 4);
    q.alloc((size_t)rows * m->q_heads * D * 4);
    attn.alloc((size_t)rows * m->q_heads * D * 4);
    hidden.alloc((size_t)rows * std::max(m->ffn_rows, 1) * 4);
    logits.alloc((size_t)rows * m->vocab_rows * 4);
    std::vector<const QMatrix*> mats;
    for (const auto& L : m->layers) {
      mats.push_back(&L.qkv);
      mats.push_back(&L.wo);
      mats.push_back(&L.gateup);
      mats.push_back(&L.down);
    }
    mats.push_back(&m->lm_head);
    int chunks = 1, cnt = 1;
    size_t parts = 1;
    const int grid = sm_count(m->device);
    for (const QMatrix* mm : mats) {
      if (!tc_gemm_ok(*mm, rows))
        invalid("batched decode: every projection must be Q8_0, Q4_0 or Q4_1");
      chunks = std::max(chunks, mm->nchunks);
      cnt = std::max(cnt, tc_counter_count(*mm));
      parts = std::max(parts, tc_partial_floats(*mm, rows, grid));
    }
    staged.alloc((size_t)chunks * tc_chunk_bytes(tc_mp(rows)));
    tc_parts.alloc(parts * 4);
    tc_cnt.alloc((size_t)cnt * 4);
    zero_now(tc_cnt.p, tc_cnt.bytes);
    status.alloc(sizeof(DeviceStatus));
    zero_now(status.p, status.bytes);
    tcws.partials = tc_parts.as<float>();
    tcws.partial_floats = parts;
    tcws.counters = tc_cnt.as<int>();
    tcws.counter_count = cnt;
    tcws.status = status.as<DeviceStatus>();
    attn_check_tiled(m->q_heads, m->kv_heads, D);
    // (KV head, split, row) CTAs for about four waves of two per SM at the
    // longest context, at least 64 positions per split
    attn_nsplit = std::max(1, std::min((8 * grid + rows * m->kv_heads - 1) / (rows * m->kv_heads),
                                       (c.max_seq_len + 63) / 64));
    attn_ws.alloc(attn_ws_floats(m->q_heads, m->kv_heads, D, attn_nsplit) * rows * 4);
    attn_cnt.alloc((size_t)rows * m->kv_heads * 4);
    zero_now(attn_cnt.p, attn_cnt.bytes);
    rows_dev.alloc((size_t)3 * rows * 4);
    zero_now(rows_dev.p, rows_dev.bytes);
    keys_dev.alloc((size_t)rows * 8);
    zero_now(keys_dev.p, keys_dev.bytes);
    step_dev.alloc(4);
    zero_now(step_dev.p, 4);
  }

  // The kernels of one pass of `rows` rows on stream s (rows_dev filled).
  // keys/values: the first sequence's cache, sequences seq_stride elements
  // apart, fp32 or (kv_bf16) bf16 elements. Returns the number of kernels
  // launched.
  int record(int rows, void* keys, void* values, long long seq_stride, bool kv_bf16,
             cudaStream_t s) {
    const mlb_config& c = m->cfg;
    const int D = c.head_dim;
    const size_t layer_kv = (size_t)c.max_seq_len * m->kv_heads * D;
    const bool tp = m->tp_size > 1;
    int launches = 0;
    const size_t esz = kv_bf16 ? 2 : 4;
    // layer l's base of the first sequence's cache, typed as the kernels take it
    auto kv_at = [&](void* base, int l) {
      return reinterpret_cast<float*>(static_cast<uint8_t*>(base) + (size_t)l * layer_kv * esz);
    };
    auto stage = [&](const float* src, int ld, int k, int chunks, const float* norm) {
      tc_stage_launch(src, ld, rows, k, chunks, norm, c.rms_norm_eps, nullptr,
                      staged.as<uint8_t>(), s, true);
      ++launches;
    };
    auto gemm = [&](const QMatrix& w, const BEpi& e) {
      tc_gemm_launch(w, staged.as<uint8_t>(), rows, e, tcws, s, 0, true);
      ++launches;
    };
    gather_rows_kernel<<<dim3((c.dim + 255) / 256, rows), 256, 0, s>>>(
        x.as<float>(), m->embedding.as<float>(), tok(), rows, c.dim);
    MLB_CUDA(cudaGetLastError());
    ++launches;
    for (int l = 0; l < c.n_layers; ++l) {
      const LayerPlan& L = m->layers[l];
      stage(x.as<float>(), c.dim, c.dim, L.qkv.nchunks, L.attn_norm.as<float>());
      BEpi e{};
      e.kind = kEpiQkv;
      e.q_rows = m->q_heads * D;
      e.kv_rows = m->kv_heads * D;
      e.k_off = L.qkv_k_off;
      e.v_off = L.qkv_v_off;
      e.head_dim = D;
      e.neox = m->neox;
      e.bias = L.bias.p ? L.bias.as<float>() : nullptr;
      e.rope = m->rope.as<float2>();
      e.row_pos = pos();
      e.row_seq = seq();
      e.keys = kv_at(keys, l);
      e.values = kv_at(values, l);
      e.seq_stride = seq_stride;
      e.kv_bf16 = kv_bf16;
      e.q_out = q.as<float>();
      gemm(L.qkv, e);

      AttnLaunch al;
      al.q = q.as<float>();
      al.keys = kv_at(keys, l);
      al.values = kv_at(values, l);
      al.kv_bf16 = kv_bf16;
      al.H = m->q_heads;
      al.KV = m->kv_heads;
      al.D = D;
      al.nsplit = attn_nsplit;
      al.scale = attn_scale(D);
      al.include_current_v = mode == MLB_ATTN_STANDARD;
      al.ws = attn_ws.as<float>();
      al.counters = attn_cnt.as<int>();
      al.out = attn.as<float>();
      al.rows = rows;
      al.row_pos = pos();
      al.row_seq = seq();
      al.seq_stride = seq_stride;
      attn_launch(al, s, true);
      ++launches;

      const int qd = m->q_heads * D;
      stage(attn.as<float>(), qd, qd, L.wo.nchunks, nullptr);
      BEpi eo{};
      if (!tp) {
        eo.kind = kEpiResidual;
        eo.y = x2.as<float>();
        eo.resid = x.as<float>();
        eo.ldy = eo.ldr = c.dim;
        eo.n_out = c.dim;
        gemm(L.wo, eo);
      } else {
        eo.kind = kEpiStore;
        eo.y = tmp.as<float>();
        eo.ldy = c.dim;
        eo.n_out = c.dim;
        gemm(L.wo, eo);
        nccl_check(ncclAllReduce(tmp.p, tmp.p, (size_t)rows * c.dim, ncclFloat, ncclSum, m->comm, s),
                   "ncclAllReduce");
        op_add(x.as<float>(), tmp.as<float>(), rows * c.dim, x2.as<float>(), s);
        ++launches;
      }

      stage(x2.as<float>(), c.dim, c.dim, L.gateup.nchunks, L.ffn_norm.as<float>());
      BEpi eg{};
      eg.kind = kEpiSwiglu;
      eg.y = hidden.as<float>();
      eg.ldy = m->ffn_rows;
      eg.n_out = m->ffn_rows;
      gemm(L.gateup, eg);

      stage(hidden.as<float>(), m->ffn_rows, m->ffn_rows, L.down.nchunks, nullptr);
      BEpi ed{};
      if (!tp) {
        ed.kind = kEpiResidual;
        ed.y = x.as<float>();
        ed.resid = x2.as<float>();
        ed.ldy = ed.ldr = c.dim;
        ed.n_out = c.dim;
        gemm(L.down, ed);
      } else {
        ed.kind = kEpiStore;
        ed.y = tmp.as<float>();
        ed.ldy = c.dim;
        ed.n_out = c.dim;
        gemm(L.down, ed);
        nccl_check(ncclAllReduce(tmp.p, tmp.p, (size_t)rows * c.dim, ncclFloat, ncclSum, m->comm, s),
                   "ncclAllReduce");
        op_add(x2.as<float>(), tmp.as<float>(), rows * c.dim, x.as<float>(), s);
        ++launches;
      }
    }
    stage(x.as<float>(), c.dim, c.dim, m->lm_head.nchunks, m->final_norm.as<float>());
    BEpi el{};
    el.kind = kEpiStore;
    el.y = logits.as<float>();
    el.ldy = m->vocab_rows;
    el.n_out = m->vocab_rows;
    el.argmax_keys = keys_dev.as<unsigned long long>();
    el.argmax_base = m->vocab_row0;
    gemm(m->lm_head, el);
    if (tp)
      nccl_check(ncclAllReduce(keys_dev.p, keys_dev.p, (size_t)rows, ncclUint64, ncclMax, m->comm, s),
                 "ncclAllReduce");
    return launches;
  }

  void check_status() {
    DeviceStatus st{};
    MLB_CUDA(cudaMemcpy(&st, status.p, sizeof(st), cudaMemcpyDeviceToHost));
    if (st.code != 0) {
      zero_now(tc_cnt.p, tc_cnt.bytes);
      zero_now(attn_cnt.p, attn_cnt.bytes);
      zero_now(keys_dev.p, keys_dev.bytes);
      zero_now(status.p, sizeof(st));
      fail(st.code, "batched step: a device-side check failed (site " + std::to_string(st.where) +
                        ")");
    }
  }
};

constexpr int kDecodeChunk = 1024;  // decode steps per token record

struct BatchImpl {
  ModelImpl* m = nullptr;
  int n_seqs = 0;
  cudaStream_t stream = nullptr;
  DevBuf keys, values;  // [n_seqs][L][S][KV_local][D], fp32 or bf16 elements
  long long seq_stride = 0;  // elements
  bool kv_bf16 = false;
  BatchEngine eng;
  int* h_rows = nullptr;       // pinned [3][64]
  int* h_out = nullptr;        // pinned decode tokens
  size_t h_out_cap = 0;
  DevBuf out_dev;              // decode tokens [steps][n_seqs]
  cudaGraphExec_t exec = nullptr;
  int kernels_per_step = 0;
  ~BatchImpl() {
    if (m) cudaSetDevice(m->device);
    if (stream) cudaStreamSynchronize(stream);
    if (exec) cudaGraphExecDestroy(exec);
    if (h_rows) cudaFreeHost(h_rows);
    if (h_out) cudaFreeHost(h_out);
    if (stream) cudaStreamDestroy(stream);
  }
};

// Validates rows of (sequence, token, position) against the model and the
// sequential semantics of ForwardBatch: rows of one sequence in strictly
// increasing position order.
static void validate_rows(const ModelImpl& m, int n_seqs, int n, const int* seqs, const int* toks,
                          const int* poss) {
  if (n <= 0) invalid("ForwardBatch: empty batch");
  std::vector<int> last(n_seqs, -1);
  for (int i = 0; i < n; ++i) {
    const int s = seqs ? seqs[i] : 0;
    if (s < 0 || s >= n_seqs) out_of_range("ForwardBatch: sequence id out of range");
    if (toks[i] < 0 || toks[i] >= m.cfg.vocab_size) out_of_range("ForwardToken token id out of range");
    if (poss[i] < 0 || poss[i] >= m.cfg.max_seq_len) out_of_range("ForwardToken position out of range");
    if (poss[i] <= last[s])
      invalid("ForwardBatch: rows of one sequence need strictly increasing positions");
    last[s] = poss[i];
  }
}

BatchImpl* batch_create(ModelImpl& m, int n_seqs, int mode, int kv_type) {
  if (!m.finalized) invalid("mlb_batch_create: model is not finalized");
  if (n_seqs < 1 || n_seqs > kTcMaxMp)
    invalid("mlb_batch_create: 1 to " + std::to_string(kTcMaxMp) + " sequences");
  if (mode != MLB_ATTN_CPU_COMPAT && mode != MLB_ATTN_STANDARD)
    invalid("mlb_batch_create: unknown attention mode");
  if (kv_type != MLB_KV_F32 && kv_type != MLB_KV_BF16)
    invalid("mlb_batch_create: unknown KV cache type");
  const mlb_config& c0 = m.cfg;
  const int g = m.q_heads / std::max(m.kv_heads, 1);
  if (kv_type == MLB_KV_BF16 &&
      (c0.head_dim % 4 != 0 || c0.head_dim > 128 || (g != 1 && g != 2 && g != 4 && g != 8)))
    invalid("mlb_batch_create: a bf16 KV cache needs head_dim a multiple of 4 up to 128 and 1, "
            "2, 4 or 8 query heads per KV head");
  set_device(m.device);
  auto b = std::make_unique<BatchImpl>();
  b->m = &m;
  b->n_seqs = n_seqs;
  MLB_CUDA(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
  const mlb_config& c = m.cfg;
  b->seq_stride = (long long)c.n_layers * c.max_seq_len * m.kv_heads * c.head_dim;
  b->kv_bf16 = kv_type == MLB_KV_BF16;
  const size_t kv = (size_t)n_seqs * b->seq_stride * (b->kv_bf16 ? 2 : 4);
  b->keys.alloc(kv);
  b->values.alloc(kv);
  zero_now(b->keys.p, kv);
  zero_now(b->values.p, kv);
  b->eng.init(&m, n_seqs, mode);
  MLB_CUDA(cudaMallocHost(&b->h_rows, 3 * kTcMaxMp * sizeof(int)));
  return b.release();
}

void batch_destroy(BatchImpl* b) { delete b; }

void batch_reset(BatchImpl& b) {
  set_device(b.m->device);
  MLB_CUDA(cudaMemsetAsync(b.keys.p, 0, b.keys.bytes, b.stream));
  MLB_CUDA(cudaMemsetAsync(b.values.p, 0, b.values.bytes, b.stream));
  MLB_CUDA(cudaStreamSynchronize(b.stream));
}

// Seeded K/V rows [0, n_pos) of one sequence (the values mlb_context_fill_kv writes).
void fill_kv_rows(void* keys, void* values, bool bf16, const ModelImpl& m, int n_pos,
                  uint64_t seed, float scale, cudaStream_t s);

void batch_fill_kv(BatchImpl& b, int seq, int n_pos, uint64_t seed, float scale) {
  if (seq < 0 || seq >= b.n_seqs) out_of_range("mlb_batch_fill_kv: sequence id out of range");
  if (n_pos < 0 || n_pos > b.m->cfg.max_seq_len) out_of_range("mlb_batch_fill_kv: n_pos out of range");
  set_device(b.m->device);
  const size_t off = (size_t)seq * b.seq_stride * (b.kv_bf16 ? 2 : 4);
  fill_kv_rows(b.keys.as<uint8_t>() + off, b.values.as<uint8_t>() + off, b.kv_bf16, *b.m, n_pos,
               seed, scale, b.stream);
  MLB_CUDA(cudaStreamSynchronize(b.stream));
}

// Copies the logits of `rows` rows (this rank's vocabulary rows, or all ranks'
// under tensor parallelism) into host memory [rows][vocab].
static void rows_logits_to_host(BatchEngine& e, int rows, float* out, cudaStream_t s) {
  ModelImpl& m = *e.m;
  const int V = m.cfg.vocab_size, vr = m.vocab_rows;
  std::vector<float> buf;
  if (m.tp_size == 1) {
    MLB_CUDA(cudaMemcpyAsync(out, e.logits.p, (size_t)rows * V * 4, cudaMemcpyDeviceToHost, s));
    MLB_CUDA(cudaStreamSynchronize(s));
    return;
  }
  DevBuf all((size_t)m.tp_size * rows * vr * 4);
  nccl_check(ncclAllGather(e.logits.p, all.p, (size_t)rows * vr, ncclFloat, m.comm, s),
             "ncclAllGather");
  buf.resize((size_t)m.tp_size * rows * vr);
  MLB_CUDA(cudaMemcpyAsync(buf.data(), all.p, buf.size() * 4, cudaMemcpyDeviceToHost, s));
  MLB_CUDA(cudaStreamSynchronize(s));
  for (int rk = 0; rk < m.tp_size; ++rk)
    for (int r = 0; r < rows; ++r)
      std::memcpy(out + (size_t)r * V + (size_t)rk * vr, buf.data() + ((size_t)rk * rows + r) * vr,
                  (size_t)vr * 4);
}

// One pass over host rows; greedy ids (and optionally the logits) to host.
static void engine_forward(BatchEngine& e, int n, const int* seqs, const int* toks, const int* poss,
                           void* keys, void* values, long long seq_stride, bool kv_bf16,
                           int* h_rows, float* logits_host, int* next_host, cudaStream_t s) {
  const int R = e.max_rows;
  for (int i = 0; i < n; ++i) {
    h_rows[i] = toks[i];
    h_rows[R + i] = poss[i];
    h_rows[2 * R + i] = seqs ? seqs[i] : 0;
  }
  MLB_CUDA(cudaMemcpyAsync(e.rows_dev.p, h_rows, (size_t)3 * R * 4, cudaMemcpyHostToDevice, s));
  e.record(n, keys, values, seq_stride, kv_bf16, s);
  std::vector<unsigned long long> kh(n);
  MLB_CUDA(cudaMemcpyAsync(kh.data(), e.keys_dev.p, (size_t)n * 8, cudaMemcpyDeviceToHost, s));
  MLB_CUDA(cudaMemsetAsync(e.keys_dev.p, 0, (size_t)n * 8, s));
  MLB_CUDA(cudaStreamSynchronize(s));
  e.check_status();
  if (next_host)
    for (int i = 0; i < n; ++i) {
      const unsigned long long k = kh[i];
      next_host[i] = k == 0ull ? 0 : (int)(0xFFFFFFFFu - (unsigned int)(k & 0xFFFFFFFFull));
    }
  if (logits_host) rows_logits_to_host(e, n, logits_host, s);
}

void batch_forward(BatchImpl& b, int n, const int* seqs, const int* toks, const int* poss,
                   float* logits_host, int* next_host) {
  if (n > b.eng.max_rows)
    invalid("mlb_batch_forward: at most " + std::to_string(b.eng.max_rows) + " rows per call");
  validate_rows(*b.m, b.n_seqs, n, seqs, toks, poss);
  set_device(b.m->device);
  engine_forward(b.eng, n, seqs, toks, poss, b.keys.p, b.values.p, b.seq_stride, b.kv_bf16,
                 b.h_rows, logits_host, next_host, b.stream);
}

// Greedy decode of every sequence in lockstep: row r = sequence r, one pass
// per step captured once in a CUDA graph (with the step's finalize kernel),
// tokens and positions advanced on the device.
void batch_decode_greedy(BatchImpl& b, const int* toks, const int* poss, int steps, int* out_host) {
  if (steps < 0) invalid("mlb_batch_decode_greedy: negative step count");
  if (steps == 0) return;
  const int n = b.n_seqs;
  std::vector<int> seqs(n);
  for (int i = 0; i < n; ++i) {
    seqs[i] = i;
    if (poss[i] + steps > b.m->cfg.max_seq_len) out_of_range("ForwardToken position out of range");
  }
  validate_rows(*b.m, b.n_seqs, n, seqs.data(), toks, poss);
  set_device(b.m->device);
  BatchEngine& e = b.eng;
  const int R = e.max_rows;
  for (int i = 0; i < n; ++i) {
    b.h_rows[i] = toks[i];
    b.h_rows[R + i] = poss[i];
    b.h_rows[2 * R + i] = i;
  }
  MLB_CUDA(cudaMemcpyAsync(e.rows_dev.p, b.h_rows, (size_t)3 * R * 4, cudaMemcpyHostToDevice,
                           b.stream));
  if (!b.h_out) {
    // a fixed token record of kDecodeChunk steps: the graph captures its
    // address once, longer decodes run in chunks of it
    b.h_out_cap = (size_t)kDecodeChunk * n;
    MLB_CUDA(cudaMallocHost(&b.h_out, b.h_out_cap * 4));
    b.out_dev.alloc(b.h_out_cap * 4);
  }
  if (!b.exec) {
    cudaGraph_t g = nullptr;
    MLB_CUDA(cudaStreamBeginCapture(b.stream, cudaStreamCaptureModeThreadLocal));
    int k = 0;
    try {
      k = e.record(n, b.keys.p, b.values.p, b.seq_stride, b.kv_bf16, b.stream);
      batch_finalize_kernel<<<1, 64, 0, b.stream>>>(e.keys_dev.as<unsigned long long>(), e.tok(),
                                                    e.pos(), n, b.out_dev.as<int>(),
                                                    e.step_dev.as<int>());
    } catch (...) {
      cudaStreamEndCapture(b.stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    MLB_CUDA(cudaStreamEndCapture(b.stream, &g));
    cudaError_t err = cudaGraphInstantiate(&b.exec, g, 0);
    cudaGraphDestroy(g);
    MLB_CUDA(err);
    b.kernels_per_step = k + 1;
  }
  for (int s0 = 0; s0 < steps; s0 += kDecodeChunk) {
    const int k = std::min(kDecodeChunk, steps - s0);
    MLB_CUDA(cudaMemsetAsync(e.step_dev.p, 0, 4, b.stream));
    for (int i = 0; i < k; ++i) MLB_CUDA(cudaGraphLaunch(b.exec, b.stream));
    MLB_CUDA(cudaMemcpyAsync(b.h_out, b.out_dev.p, (size_t)k * n * 4, cudaMemcpyDeviceToHost,
                             b.stream));
    MLB_CUDA(cudaStreamSynchronize(b.stream));
    e.check_status();
    std::memcpy(out_host + (size_t)s0 * n, b.h_out, (size_t)k * n * 4);
  }
}

// ForwardBatch on a single context: its tokens at their positions in passes
// of up to 64 rows; the logits of the last token to host.
void context_forward_batch(ContextImpl& c, int n, const int* toks, const int* poss, float* logits_host) {
  validate_rows(*c.m, 1, n, nullptr, toks, poss);
  set_device(c.m->device);
  if (!c.batch) {
    c.batch = new BatchEngine();
    c.batch->init(c.m, kTcMaxMp, c.attention_mode);
  }
  MLB_CUDA(cudaStreamSynchronize(c.stream));
  std::vector<int> rows(3 * kTcMaxMp, 0);
  std::vector<float> last;
  const int V = c.m->cfg.vocab_size;
  for (int i0 = 0; i0 < n; i0 += kTcMaxMp) {
    const int k = std::min(kTcMaxMp, n - i0);
    const bool tail = i0 + k == n;
    if (tail) last.resize((size_t)k * V);
    engine_forward(*c.batch, k, nullptr, toks + i0, poss + i0, c.keys.p, c.values.p, 0, c.kv_bf16,
                   rows.data(), tail ? last.data() : nullptr, nullptr, c.stream);
  }
  std::memcpy(logits_host, last.data() + (last.size() - V), (size_t)V * 4);
}

void batch_engine_free(BatchEngine* e) { delete e; }

int batch_kernels_per_step(const BatchImpl& b) { return b.kernels_per_step; }
cudaStream_t batch_stream(const BatchImpl& b) { return b.stream; }

}  // namespace mlb

// gguf.cu — GGUF model files loaded straight into device memory.
//
// Reference: LoadGgufModel (src/gguf_loader.cc:302-418) parses the file with
// GgufReader::Load (src/gguf.cc:420-600), builds the ModelConfig from the
// metadata (BuildConfig, src/gguf_loader.cc:13-88), maps tensor names
// (MapTensorName, :91-160), reads every tensor into a std::vector
// (ReadGgufTensorRaw, src/gguf.cc:655-693), dequantises norms, biases and the
// embedding to F32 (load_f32, :350-372) and keeps linear weights as GGUF
// blocks; UploadModelWeightsToCuda (src/model.cc:345-374) then cudaMallocs
// and copies each weight from pageable memory.
//
// Here the file is memory-mapped once. Each tensor's shard (this rank's rows)
// moves through two pinned staging buffers: host threads copy the next piece
// out of the page cache while the previous one is in flight to the device
// (cudaMemcpyAsync), so no tensor is held in host memory and the copies run
// at pinned-DMA speed. Norms, biases and the embedding stored quantised or as
// F16 are converted to F32 on the device with the reference's arithmetic
// (DequantizeFromQ80/Q40/Q41, src/quant.cc:170-361; F16 exactly). F16 linear
// weights, which the reference rejects (LoadQuantizedTensor,
// src/gguf_loader.cc:238-240), are accepted and widened to F32 (exact).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <unordered_set>
#include <vector>

#include "runtime.cuh"

namespace mlb {

namespace {

// GGUF value types (the GGUF format; src/gguf.h:20-34 names them).
enum : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32v = 6, kBool = 7,
  kStr = 8, kArr = 9, kU64 = 10, kI64 = 11, kF64 = 12
};
// ggml tensor types read here.
enum : uint32_t { kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ40 = 2, kGgmlQ41 = 3, kGgmlQ80 = 8 };
constexpr uint64_t kDefaultAlignment = 32;

struct MetaValue {
  uint32_t type = 0;
  bool is_int = false, is_float = false;
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  uint32_t arr_type = 0;
  uint64_t arr_len = 0;
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // GGUF order: dims[0] is the row length
  uint32_t type = 0;
  uint64_t offset = 0;
};

// Bounds-checked little-endian reads over the mapped file.
struct Cursor {
  const uint8_t* p;
  uint64_t size, pos = 0;
  template <class T>
  bool get(T& v) {
    if (pos > size || size - pos < sizeof(T)) return false;
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return true;
  }
  bool str(std::string& s) {
    uint64_t n = 0;
    if (!get(n) || n > size - pos) return false;
    s.assign(reinterpret_cast<const char*>(p + pos), n);
    pos += n;
    return true;
  }
  bool skip(uint64_t n) {
    if (n > size - pos) return false;
    pos += n;
    return true;
  }
};

uint64_t scalar_bytes(uint32_t t) {
  switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32v: return 4;
    case kU64: case kI64: case kF64: return 8;
  }
  return 0;
}

bool read_value(Cursor& c, uint32_t type, MetaValue& v, int depth = 0) {
  v.type = type;
  switch (type) {
    case kU8: { uint8_t x; if (!c.get(x)) return false; v.i = x; v.is_int = true; return true; }
    case kI8: { int8_t x; if (!c.get(x)) return false; v.i = x; v.is_int = true; return true; }
    case kU16: { uint16_t x; if (!c.get(x)) return false; v.i = x; v.is_int = true; return true; }
    case kI16: { int16_t x; if (!c.get(x)) return false; v.i = x; v.is_int = true; return true; }
    case kU32: { uint32_t x; if (!c.get(x)) return false; v.i = x; v.is_int = true; return true; }
    case kI32: { int32_t x; if (!c.get(x)) return false; v.i = x; v.is_int = true; return true; }
    case kU64: { uint64_t x; if (!c.get(x)) return false; v.i = (int64_t)x; v.is_int = true; return true; }
    case kI64: { int64_t x; if (!c.get(x)) return false; v.i = x; v.is_int = true; return true; }
    case kF32v: { float x; if (!c.get(x)) return false; v.f = x; v.is_float = true; return true; }
    case kF64: { double x; if (!c.get(x)) return false; v.f = x; v.is_float = true; return true; }
    case kBool: { uint8_t x; if (!c.get(x)) return false; v.i = x; return true; }
    case kStr: return c.str(v.s);
    case kArr: {
      if (depth > 0) return false;  // nested arrays are not used by model files
      if (!c.get(v.arr_type) || !c.get(v.arr_len)) return false;
      if (v.arr_type == kStr) {
        for (uint64_t k = 0; k < v.arr_len; ++k) {
          uint64_t n = 0;
          if (!c.get(n) || !c.skip(n)) return false;
        }
        return true;
      }
      const uint64_t eb = scalar_bytes(v.arr_type);
      if (eb == 0 || v.arr_len > (c.size - c.pos) / eb) return false;
      return c.skip(eb * v.arr_len);
    }
  }
  return false;
}

}  // namespace

// A parsed GGUF file kept memory-mapped (GgufReader, src/gguf.h:56-68).
struct GgufFile {
  std::string path;
  int fd = -1;
  const uint8_t* base = nullptr;
  uint64_t size = 0;
  uint32_t version = 0;
  std::map<std::string, MetaValue> meta;
  std::vector<TensorInfo> tensors;
  uint64_t data_offset = 0;

  ~GgufFile() {
    if (base) munmap(const_cast<uint8_t*>(base), size);
    if (fd >= 0) close(fd);
  }

  [[noreturn]] void bad(const std::string& why) const { invalid("GGUF parse error: " + why); }

  void open_and_parse(const std::string& p) {
    path = p;
    fd = ::open(p.c_str(), O_RDONLY);
    if (fd < 0) bad("cannot open " + p);
    struct stat st {};
    if (fstat(fd, &st) != 0) bad("cannot stat " + p);
    size = (uint64_t)st.st_size;
    if (size < 24) bad("invalid GGUF magic");
    void* m = mmap(nullptr, size, PROT_READ, MAP_SHARED, fd, 0);
    if (m == MAP_FAILED) bad("cannot map " + p);
    base = static_cast<const uint8_t*>(m);
    Cursor c{base, size};
    if (std::memcmp(base, "GGUF", 4) != 0) bad("invalid GGUF magic");
    c.pos = 4;
    c.get(version);
    if (version != 3) bad("unsupported GGUF version: " + std::to_string(version));
    uint64_t n_tensors = 0, n_meta = 0;
    if (!c.get(n_tensors) || !c.get(n_meta)) bad("failed to read header counts");
    if (n_tensors > (1u << 20)) bad("too many tensors: " + std::to_string(n_tensors));
    if (n_meta > (1u << 20)) bad("too many metadata entries: " + std::to_string(n_meta));
    for (uint64_t i = 0; i < n_meta; ++i) {
      std::string key;
      uint32_t type = 0;
      if (!c.str(key)) bad("failed to read metadata key at index " + std::to_string(i));
      if (meta.count(key)) bad("duplicate metadata key: " + key);
      if (!c.get(type)) bad("failed to read metadata type for key: " + key);
      MetaValue v;
      if (!read_value(c, type, v)) bad("failed to read metadata value for key: " + key);
      meta.emplace(key, std::move(v));
    }
    std::unordered_set<std::string> names;
    tensors.reserve(n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
      TensorInfo t;
      uint32_t nd = 0;
      if (!c.str(t.name)) bad("failed to read tensor name at index " + std::to_string(i));
      if (!c.get(nd) || nd == 0 || nd > 4) bad("invalid tensor n_dims for: " + t.name);
      t.dims.resize(nd);
      for (uint32_t d = 0; d < nd; ++d)
        if (!c.get(t.dims[d]) || t.dims[d] == 0)
          bad("invalid zero tensor dimension for: " + t.name);
      if (!c.get(t.type) || !c.get(t.offset)) bad("failed to read tensor type for: " + t.name);
      if (!names.insert(t.name).second) bad("duplicate tensor name: " + t.name);
      tensors.push_back(std::move(t));
    }
    uint64_t align = kDefaultAlignment;
    auto it = meta.find("general.alignment");
    if (it != meta.end()) {
      if (!it->second.is_int || it->second.i <= 0 || (it->second.i & (it->second.i - 1)) != 0)
        bad("invalid general.alignment");
      align = (uint64_t)it->second.i;
    }
    data_offset = (c.pos + align - 1) / align * align;
    if (data_offset > size) bad("GGUF file ended before tensor data section");
    for (const TensorInfo& t : tensors) {
      const uint64_t n = bytes_of(t);
      if (n == 0) bad("invalid tensor data size for: " + t.name);
      if (t.offset > size - data_offset || n > size - data_offset - t.offset)
        bad("tensor data out of file bounds for: " + t.name);
    }
  }

  static uint64_t numel(const TensorInfo& t) {
    uint64_t n = 1;
    for (uint64_t d : t.dims) n *= d;
    return n;
  }
  // Bytes of a tensor's data (0 when the type is not one read here).
  static uint64_t bytes_of(const TensorInfo& t) {
    const uint64_t n = numel(t);
    switch (t.type) {
      case kGgmlF32: return n * 4;
      case kGgmlF16: return n * 2;
      case kGgmlQ40: return (n + 31) / 32 * 18;
      case kGgmlQ41: return (n + 31) / 32 * 20;
      case kGgmlQ80: return (n + 31) / 32 * 34;
    }
    return 1;  // unknown types are rejected when a weight needs them
  }

  bool get_int(const std::string& k, int64_t& out) const {
    auto it = meta.find(k);
    if (it == meta.end() || !it->second.is_int) return false;
    out = it->second.i;
    return true;
  }
  bool get_float(const std::string& k, double& out) const {
    auto it = meta.find(k);
    if (it == meta.end() || !it->second.is_float) return false;
    out = it->second.f;
    return true;
  }
};

// BuildConfig (src/gguf_loader.cc:13-88): qwen2.* keys, else llama.* keys,
// else 0; NeoX RoPE for general.architecture == "qwen2"; the vocabulary size
// is the length of tokenizer.ggml.tokens; head_dim = dim / n_heads.
mlb_config gguf_config(const GgufFile& g) {
  mlb_config c{};
  auto u32 = [&](const char* key, int fb) {
    int64_t v = 0;
    return g.get_int(std::string("qwen2.") + key, v) || g.get_int(std::string("llama.") + key, v)
               ? (int)v
               : fb;
  };
  auto f32 = [&](const char* key, float fb) {
    double v = 0.0;
    return g.get_float(std::string("qwen2.") + key, v) ||
                   g.get_float(std::string("llama.") + key, v)
               ? (float)v
               : fb;
  };
  auto arch = g.meta.find("general.architecture");
  c.rope_type = (arch != g.meta.end() && arch->second.type == kStr && arch->second.s == "qwen2") ? 1 : 0;
  c.n_layers = u32("block_count", 0);
  c.dim = u32("embedding_length", 0);
  c.hidden_dim = u32("feed_forward_length", 0);
  c.n_heads = u32("attention.head_count", 0);
  c.n_kv_heads = u32("attention.head_count_kv", 0);
  c.max_seq_len = u32("context_length", 0);
  c.rope_theta = f32("rope.freq_base", 0.0f);
  c.rms_norm_eps = f32("attention.layer_norm_rms_epsilon", 0.0f);
  auto tok = g.meta.find("tokenizer.ggml.tokens");
  if (tok != g.meta.end() && tok->second.type == kArr && tok->second.arr_type == kStr)
    c.vocab_size = (int)tok->second.arr_len;
  if (c.n_layers <= 0 || c.dim <= 0 || c.hidden_dim <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
      c.max_seq_len <= 0 || c.vocab_size <= 0)
    invalid("Failed to build config: Invalid model config from GGUF: dim=" + std::to_string(c.dim) +
            " layers=" + std::to_string(c.n_layers) + " heads=" + std::to_string(c.n_heads) +
            " vocab=" + std::to_string(c.vocab_size));
  if (c.dim % c.n_heads != 0) invalid("Failed to build config: dim not divisible by n_heads");
  if (c.n_heads % c.n_kv_heads != 0)
    invalid("Failed to build config: n_heads not divisible by n_kv_heads");
  c.head_dim = c.dim / c.n_heads;
  return c;
}

// MapTensorName (src/gguf_loader.cc:91-160) as (kind, layer); kind < 0 for
// names the model does not use.
static void map_tensor(const std::string& n, int* kind, int* layer) {
  *kind = -1;
  *layer = -1;
  if (n == "token_embd.weight") { *kind = MLB_W_TOKEN_EMBEDDING; return; }
  if (n == "output_norm.weight") { *kind = MLB_W_FINAL_NORM; return; }
  if (n == "output.weight") { *kind = MLB_W_LM_HEAD; return; }
  if (n.rfind("blk.", 0) != 0) return;
  const size_t d1 = n.find('.', 4);
  if (d1 == std::string::npos) return;
  const size_t d2 = n.find('.', d1 + 1);
  if (d2 == std::string::npos) return;
  const std::string ls = n.substr(4, d1 - 4), op = n.substr(d1 + 1, d2 - d1 - 1),
                    suffix = n.substr(d2 + 1);
  if (ls.empty() || ls.find_first_not_of("0123456789") != std::string::npos || ls.size() > 6) return;
  static const std::map<std::string, int> weights = {
      {"attn_norm", MLB_W_ATTENTION_NORM}, {"attn_q", MLB_W_WQ},     {"attn_k", MLB_W_WK},
      {"attn_v", MLB_W_WV},                {"attn_output", MLB_W_WO}, {"ffn_norm", MLB_W_FFN_NORM},
      {"ffn_gate", MLB_W_GATE},            {"ffn_up", MLB_W_UP},     {"ffn_down", MLB_W_DOWN}};
  static const std::map<std::string, int> biases = {
      {"attn_q", MLB_W_BQ}, {"attn_k", MLB_W_BK}, {"attn_v", MLB_W_BV}};
  const auto& table = suffix == "bias" ? biases : weights;
  if (suffix != "bias" && suffix != "weight") return;
  auto it = table.find(op);
  if (it == table.end()) return;
  *kind = it->second;
  *layer = std::stoi(ls);
}

// ------------------------------------------------------ device side

namespace {

// out[i] = the F32 value of element i of a GGUF tensor stored as `type`, with
// the reference's arithmetic: F16 exactly (Fp16ToFloat, src/quant.cc:53-84),
// Q8_0 d * q, Q4_0 d * (q - 8), Q4_1 d * q + m (a rounded product, then a
// rounded sum; DequantizeFromQ80/Q40/Q41, src/quant.cc:170-361).
__global__ void gguf_to_f32_kernel(const uint8_t* src, uint32_t type, long long n, float* out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float v = 0.0f;
    if (type == kGgmlF16) {
      v = __half2float(__ushort_as_half(reinterpret_cast<const unsigned short*>(src)[i]));
    } else {
      const long long b = i >> 5;
      const int j = (int)(i & 31);
      if (type == kGgmlQ80) {
        const uint8_t* blk = src + b * 34;
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk)));
        v = __fmul_rn(d, (float)(int8_t)blk[2 + j]);
      } else {
        const int hd = type == kGgmlQ41 ? 4 : 2;
        const uint8_t* blk = src + b * (type == kGgmlQ41 ? 20 : 18);
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk)));
        const uint8_t byte = blk[hd + (j & 15)];
        const int q = j < 16 ? (byte & 15) : (byte >> 4);
        if (type == kGgmlQ40) {
          v = __fmul_rn(d, (float)(q - 8));
        } else {
          const float m =
              __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk + 2)));
          v = __fadd_rn(__fmul_rn(d, (float)q), m);
        }
      }
    }
    out[i] = v;
  }
}

// Host-to-device copies through two pinned staging buffers: while piece i is
// in flight, host threads fill the other buffer with piece i + 1 from the
// mapped file.
struct PinnedPipe {
  static constexpr size_t kPiece = (size_t)64 << 20;
  uint8_t* buf[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaStream_t s = nullptr;
  int next = 0;
  size_t bytes = 0;

  explicit PinnedPipe(cudaStream_t stream) : s(stream) {
    for (int i = 0; i < 2; ++i) {
      MLB_CUDA(cudaHostAlloc(&buf[i], kPiece, cudaHostAllocDefault));
      MLB_CUDA(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
    }
  }
  ~PinnedPipe() {
    if (s) cudaStreamSynchronize(s);
    for (int i = 0; i < 2; ++i) {
      if (ev[i]) cudaEventDestroy(ev[i]);
      if (buf[i]) cudaFreeHost(buf[i]);
    }
  }
  static void host_copy(uint8_t* dst, const uint8_t* src, size_t n) {
    const unsigned hw = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    const size_t per = (n + hw - 1) / hw;
    if (n < ((size_t)4 << 20) || hw == 1) {
      std::memcpy(dst, src, n);
      return;
    }
    std::vector<std::thread> th;
    for (unsigned t = 0; t < hw; ++t) {
      const size_t a = std::min(n, t * per), b = std::min(n, a + per);
      if (a < b) th.emplace_back([=] { std::memcpy(dst + a, src + a, b - a); });
    }
    for (auto& x : th) x.join();
  }
  void copy(void* dst, const uint8_t* src, size_t n) {
    for (size_t off = 0; off < n; off += kPiece) {
      const size_t len = std::min(kPiece, n - off);
      const int i = next;
      next ^= 1;
      MLB_CUDA(cudaEventSynchronize(ev[i]));  // the copy that last used buf[i] is done
      host_copy(buf[i], src + off, len);
      MLB_CUDA(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, buf[i], len,
                               cudaMemcpyHostToDevice, s));
      MLB_CUDA(cudaEventRecord(ev[i], s));
    }
    bytes += n;
  }
  void finish() { MLB_CUDA(cudaStreamSynchronize(s)); }
};

const char* type_name(uint32_t t) {
  switch (t) {
    case kGgmlF32: return "F32";
    case kGgmlF16: return "F16";
    case kGgmlQ40: return "Q4_0";
    case kGgmlQ41: return "Q4_1";
    case kGgmlQ80: return "Q8_0";
  }
  return "?";
}

int qtype_of(uint32_t t) {
  switch (t) {
    case kGgmlQ40: return MLB_Q4_0;
    case kGgmlQ41: return MLB_Q4_1;
    case kGgmlQ80: return MLB_Q8_0;
  }
  return MLB_F32;
}

}  // namespace

// Uploads every tensor the model uses from the mapped file (this rank's
// shards) and finalizes the model. Returns the bytes copied to the device.
size_t gguf_upload(ModelImpl& m, const GgufFile& g) {
  set_device(m.device);
  std::map<std::pair<int, int>, const TensorInfo*> byname;
  for (const TensorInfo& t : g.tensors) {
    int kind, layer;
    map_tensor(t.name, &kind, &layer);
    if (kind < 0) continue;
    if (kind >= 3 && layer >= m.cfg.n_layers) continue;
    byname[{kind, kind < 3 ? -1 : layer}] = &t;
  }
  PinnedPipe pipe(m.stream);
  const float* emb_dev = nullptr;  // the F32 embedding, for a tied lm_head
  auto load = [&](int kind, int layer, bool optional) {
    auto it = byname.find({kind, kind < 3 ? -1 : layer});
    const WeightSlot w = model_weight_slot(m, kind, layer);
    if (it == byname.end()) {
      if (optional) return;
      invalid("Failed to load GGUF weights: Missing tensor: " + w.name);
    }
    const TensorInfo& t = *it->second;
    if (t.type != kGgmlF32 && t.type != kGgmlF16 && t.type != kGgmlQ40 && t.type != kGgmlQ41 &&
        t.type != kGgmlQ80)
      invalid("Failed to load GGUF weights: Unsupported GGUF tensor type: " +
              std::to_string(t.type) + " (" + w.name + ")");
    // MapShape (src/gguf_loader.cc:163-178): [dims[1], dims[0]] for 2-D
    const uint64_t cols = t.dims[0], rows = t.dims.size() >= 2 ? t.dims[1] : 1;
    if (t.dims.size() > 2 || (uint64_t)w.cols != cols || (uint64_t)w.rows != rows)
      invalid("Failed to load GGUF weights: shape mismatch for " + w.name + ": file [" +
              std::to_string(rows) + ", " + std::to_string(cols) + "], model [" +
              std::to_string(w.rows) + ", " + std::to_string(w.cols) + "]");
    const bool quant = t.type == kGgmlQ40 || t.type == kGgmlQ41 || t.type == kGgmlQ80;
    if (quant && cols % 32 != 0)
      invalid("Failed to load GGUF weights: " + std::string(type_name(t.type)) + " rows of " +
              w.name + " are not whole 32-element blocks");
    const uint8_t* src = g.base + g.data_offset + t.offset;
    const uint64_t row_bytes = GgufFile::bytes_of(t) / rows;
    // the shard: rows [first, first + count), or columns for the biases
    uint64_t b0, b1, n_el;
    if (w.by_cols) {
      const uint64_t eb = t.type == kGgmlF16 ? 2 : 4;
      if (quant) {  // a quantised bias: the whole row, cut after widening
        b0 = 0;
        b1 = row_bytes;
      } else {
        b0 = (uint64_t)w.first * eb;
        b1 = b0 + (uint64_t)w.count * eb;
      }
      n_el = quant ? cols : (uint64_t)w.count;
    } else {
      b0 = (uint64_t)w.first * row_bytes;
      b1 = b0 + (uint64_t)w.count * row_bytes;
      n_el = (uint64_t)w.count * cols;
    }
    RawTensor r;
    const bool widen = t.type == kGgmlF16 || (quant && w.f32_only);
    r.qtype = widen || t.type == kGgmlF32 ? MLB_F32 : qtype_of(t.type);
    r.rows = w.by_cols ? 1 : w.count;
    r.cols = w.by_cols ? w.count : (int)cols;
    r.pitch = w.by_cols ? (size_t)w.count * 4 : gguf_row_bytes(r.qtype, (int)cols);
    r.buf.alloc(r.pitch * (size_t)r.rows);
    if (!widen) {
      pipe.copy(r.buf.p, src + b0, b1 - b0);
    } else {
      DevBuf raw(b1 - b0);
      pipe.copy(raw.p, src + b0, b1 - b0);
      const bool cut = w.by_cols && quant;  // widen the whole row, keep the shard's columns
      DevBuf wide(cut ? (size_t)cols * 4 : 0);
      float* dst = cut ? wide.as<float>() : r.buf.as<float>();
      const long long ne = (long long)n_el;
      gguf_to_f32_kernel<<<(unsigned)std::min<long long>((ne + 255) / 256, 4096), 256, 0, m.stream>>>(
          raw.as<uint8_t>(), t.type, ne, dst);
      MLB_CUDA(cudaGetLastError());
      if (cut)
        MLB_CUDA(cudaMemcpyAsync(r.buf.p, wide.as<float>() + w.first, (size_t)w.count * 4,
                                 cudaMemcpyDeviceToDevice, m.stream));
      pipe.finish();  // the temporaries are released on return
    }
    if (kind == MLB_W_TOKEN_EMBEDDING) emb_dev = r.buf.as<float>();
    model_put_raw(m, kind, layer, std::move(r));
  };
  load(MLB_W_TOKEN_EMBEDDING, -1, false);
  load(MLB_W_FINAL_NORM, -1, false);
  for (int l = 0; l < m.cfg.n_layers; ++l) {
    load(MLB_W_ATTENTION_NORM, l, false);
    load(MLB_W_WQ, l, false);
    load(MLB_W_WK, l, false);
    load(MLB_W_WV, l, false);
    load(MLB_W_BQ, l, true);
    load(MLB_W_BK, l, true);
    load(MLB_W_BV, l, true);
    load(MLB_W_WO, l, false);
    load(MLB_W_FFN_NORM, l, false);
    load(MLB_W_GATE, l, false);
    load(MLB_W_UP, l, false);
    load(MLB_W_DOWN, l, false);
  }
  if (byname.count({MLB_W_LM_HEAD, -1})) {
    load(MLB_W_LM_HEAD, -1, false);
  } else {
    // no output.weight: the lm_head is the embedding (src/gguf_loader.cc:401-406)
    const WeightSlot w = model_weight_slot(m, MLB_W_LM_HEAD, -1);
    RawTensor r;
    r.qtype = MLB_F32;
    r.rows = w.count;
    r.cols = w.cols;
    r.pitch = (size_t)w.cols * 4;
    r.buf.alloc(r.pitch * (size_t)w.count);
    MLB_CUDA(cudaMemcpyAsync(r.buf.p, emb_dev + (size_t)w.first * w.cols, r.pitch * (size_t)w.count,
                             cudaMemcpyDeviceToDevice, m.stream));
    pipe.finish();
    model_put_raw(m, MLB_W_LM_HEAD, -1, std::move(r));
  }
  pipe.finish();
  return pipe.bytes;
}

}  // namespace mlb

namespace mlb {

GgufFile* gguf_open(const char* path) {
  auto g = std::make_unique<GgufFile>();
  g->open_and_parse(path);
  return g.release();
}
void gguf_close(GgufFile* g) { delete g; }

}  // namespace mlb

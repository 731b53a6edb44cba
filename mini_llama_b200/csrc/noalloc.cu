// noalloc.cu — decode attention that allocates no device memory.
//
// mlb_attention_decode (capi.cu) allocates its split-K scratch (per-slice
// partial results and per-KV-head arrival counters) with cudaMalloc on every
// call. Some callers cannot allow that: hosts whose device memory is owned by
// their own allocator under a fixed budget, and latency-sensitive decode loops
// that cannot afford cudaMalloc/cudaFree (cudaFree synchronises the device).
// This entry point runs the same kernel with its scratch in a file-scope
// __device__ array instead. The array lives in every GPU that loads the
// library until the process exits.
//
// Host code cannot pass the array's name to a kernel (in host code the name is
// a host-side stand-in, not a device address), so the device address is looked
// up with cudaGetSymbolAddress once per device, on the first call made on that
// device, with that device current.
#include <algorithm>
#include <mutex>
#include <string>

#include "attention.cuh"

namespace mlb {

// Split-K partials: KV heads x slices x (H/KV) x (head_dim + 2) floats.
constexpr size_t kNoAllocScratchFloats = (size_t)1 << 20;  // 4 MiB
// Arrival counters, one per KV head; must be zero when a launch starts.
constexpr int kNoAllocMaxKvHeads = 1024;

struct NoAllocScratch {
  float partials[kNoAllocScratchFloats];
  int counters[kNoAllocMaxKvHeads];
};
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

static std::mutex g_noalloc_mu;
static NoAllocScratch* g_noalloc_ptr[64] = {};

// Device address of the scratch on the current device (set up on first use).
static NoAllocScratch* noalloc_scratch(int device_id) {
  if (device_id < 0 || device_id >= 64) invalid("no-alloc attention: device id out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[device_id]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      (void)cudaGetLastError();
      fail(MLB_ERR_CUDA, std::string("no-alloc attention: cudaGetSymbolAddress failed: ") +
                             cudaGetErrorString(e));
    }
    g_noalloc_ptr[device_id] = static_cast<NoAllocScratch*>(p);
  }
  return g_noalloc_ptr[device_id];
}

}  // namespace mlb

using namespace mlb;

extern "C" int mlb_attention_decode_noalloc(const float* q, const float* keys,
                                            const float* values, int n_layers, int max_seq_len,
                                            int layer, int pos, int n_heads, int n_kv_heads,
                                            int head_dim, int mode, float* out, int device_id,
                                            void* stream) {
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
    if (n_kv_heads > kNoAllocMaxKvHeads)
      invalid("no-alloc attention: n_kv_heads " + std::to_string(n_kv_heads) +
              " exceeds the fixed scratch limit of " + std::to_string(kNoAllocMaxKvHeads));
    const size_t per_split = (size_t)n_kv_heads * (n_heads / n_kv_heads) * (head_dim + 2);
    const bool tiled = attn_tiled_ok(n_heads, n_kv_heads, head_dim);
    if (tiled && per_split > kNoAllocScratchFloats)
      invalid("no-alloc attention: one split needs " + std::to_string(per_split) +
              " scratch floats, above the fixed limit of " + std::to_string(kNoAllocScratchFloats));
    set_device(device_id);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    AttnLaunch l;
    const size_t layer_off = (size_t)layer * max_seq_len * n_kv_heads * head_dim;
    l.q = q;
    l.keys = keys + layer_off;
    l.values = values + layer_off;
    l.pos_host = pos;
    l.H = n_heads;
    l.KV = n_kv_heads;
    l.D = head_dim;
    l.scale = attn_scale(head_dim);
    l.include_current_v = mode == MLB_ATTN_STANDARD;
    l.out = out;
    if (tiled) {
      NoAllocScratch* sc = noalloc_scratch(device_id);
      int nsplit = attn_splits(n_kv_heads, sm_count(device_id), pos + 1);
      nsplit = (int)std::min<size_t>((size_t)nsplit, kNoAllocScratchFloats / per_split);
      // the counters keep whatever the previous call left: start them at zero
      MLB_CUDA(cudaMemsetAsync(sc->counters, 0, (size_t)n_kv_heads * sizeof(int), s));
      l.nsplit = nsplit;
      l.ws = sc->partials;
      l.counters = sc->counters;
    }
    attn_launch(l, s, false);
  });
}

// common.cuh — error handling and sm_100a device helpers shared by the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "../../include/mlb200.h"

namespace mlb {

// ------------------------------------------------------------------ errors
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }
[[noreturn]] inline void invalid(const std::string& msg) { throw Error(MLB_ERR_INVALID, msg); }
[[noreturn]] inline void out_of_range(const std::string& msg) { throw Error(MLB_ERR_RANGE, msg); }

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw Error(MLB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
#define MLB_CUDA(call) ::mlb::check_cuda((call), #call)

void set_last_error(const std::string& msg);

// Runs f and converts exceptions into a status code + thread-local message.
template <class F>
int guarded(F&& f) {
  try {
    f();
    return MLB_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::out_of_range& e) {
    set_last_error(e.what());
    return MLB_ERR_RANGE;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return MLB_ERR_INVALID;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return MLB_ERR_INVALID;
  }
}

// Selects `device_id` for the calling thread (CudaSetDevice, src/cuda_runtime.cc).
void set_device(int device_id);

// Zeroes `bytes` of device memory and waits until it is done. cudaMemset runs
// on the legacy default stream, which the library's non-blocking streams are
// not ordered against: without the wait a large clear (a KV cache) can still
// be running when a kernel on another stream writes the same bytes.
void zero_now(void* p, size_t bytes);

// Copies host memory to the device and waits until the bytes have landed
// (cudaMemcpy from pageable memory may return before its DMA has finished, on
// the legacy stream that the library's streams are not ordered against).
void copy_to_device_now(void* dst, const void* src, size_t bytes);

// Device-side error word: kernels that give up a bounded wait record where.
struct DeviceStatus {
  int code;  // 0 = ok, else MLB_ERR_TIMEOUT
  int where;
};

// Number of SMs of the current device (cached per device).
int sm_count(int device_id);

// Launch with the programmatic-dependent-launch attribute so the kernel may
// start (and prefetch its weights) while the previous kernel on the stream
// drains; the kernel calls pdl_wait() before touching its inputs.
template <class... KArgs, class... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                cudaStream_t stream, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  MLB_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// ----------------------------------------------------------- device helpers
#if defined(__CUDACC__)

// Programmatic dependent launch: wait for the preceding grid's results /
// allow the next grid to start launching.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Four consecutive KV-cache elements as loaded (fp32: a float4; bf16: a
// uint2, widened only when used, so a prefetch does not wait for its own data)
// and as fp32. bf16 -> fp32 is exact (the high half of the fp32 bits).
template <bool BF>
struct KvRaw {
  using T = float4;
  static __device__ __forceinline__ T load(const void* p) {
    return __ldcs(static_cast<const float4*>(p));
  }
  static __device__ __forceinline__ T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ __forceinline__ float4 widen(const T& v) { return v; }
};
template <>
struct KvRaw<true> {
  using T = uint2;
  static __device__ __forceinline__ T load(const void* p) {
    return __ldcs(static_cast<const uint2*>(p));
  }
  static __device__ __forceinline__ T zero() { return make_uint2(0u, 0u); }
  static __device__ __forceinline__ float4 widen(const T& u) {
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  }
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// mbarrier helpers (shared::cta).
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: `limit` SM cycles of polling (default ~2 s), then records a
// timeout and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  DeviceStatus* status, int where,
                                                  long long limit = 4000000000LL) {
  long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > limit) {
      if (status) {
        atomicExch(&status->code, MLB_ERR_TIMEOUT);
        atomicExch(&status->where, where);
      }
      return false;
    }
  }
  return true;
}

// 16-byte asynchronous global -> shared copy (cp.async, L2 only), its group
// commit and the wait for all of this thread's groups.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Order earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned); a plain copy into this CTA only.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// D (f32 16x8) += A (f16 16x16, row) * B (f16 16x8, col). Not volatile: a pure
// function of its operands, so the compiler may interleave independent MMAs.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D (f32 16x8) = A * B with a zero accumulator input (no registers to clear).
__device__ __forceinline__ void mma_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                            uint32_t b1) {
  const float z = 0.0f;
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
  return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) {
  return *reinterpret_cast<__half2*>(&u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

#endif  // __CUDACC__

}  // namespace mlb

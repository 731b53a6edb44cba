// synth.h — seeded synthetic weights in GGUF block layout, bit-identical on
// the host (C++) and on the device (CUDA).
//
// A weight element is identified by (seed, stream, index), where stream names
// the tensor (kind * 2^20 + layer) and index is its row-major position in the
// full [rows, cols] fp32 tensor. Its value is
//     g = (sum of 12 uniform 16-bit integers - 393210) / 65536   (Irwin-Hall,
//         mean 0, variance 1; every step is integer or exact in fp32)
//     w = g * 0.02f                                          (one fp32 multiply)
// Quantised tensors are produced from these fp32 values block by block with
// the reference's quantisers (QuantizeToQ80 src/quant.cc:106-167,
// QuantizeToQ40 src/quant.cc:201-276, and for Q4_1 the reference's test
// quantiser QuantizeToQ41ForTest tests/test_cuda_quant.cc:131-188), including
// its fp16 rounding (FloatToFp16, src/quant.cc:14-50). Every float operation
// is a single IEEE-rounded multiply, add, divide or round: the device code
// uses the _rn intrinsics so nothing is contracted into an FMA, and the host
// code is compiled with -ffp-contract=off. Because of that, a tensor
// generated on the GPU (for the benchmark) has exactly the bytes the CPU
// generates (for the CPU oracles).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define MLB_HD __host__ __device__ __forceinline__
#else
#define MLB_HD inline
#endif

namespace mlb {
namespace synth {

MLB_HD uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

MLB_HD uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64(seed ^ mix64(stream + 0x632BE59BD9B4E019ull));
}

MLB_HD float fmul(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
MLB_HD float fadd(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
MLB_HD float fsub(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
MLB_HD float fdiv(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}
MLB_HD float fround(float a) {  // round half away from zero, like std::round
#if defined(__CUDA_ARCH__)
  return roundf(a);
#else
  return __builtin_roundf(a);
#endif
}
MLB_HD float fabs_(float a) { return a < 0.0f ? -a : a; }
MLB_HD uint32_t fbits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
  return u;
#endif
}
MLB_HD float bitsf(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}

// Standard-normal approximation for element `index` of a stream.
MLB_HD float gauss(uint64_t key, uint64_t index) {
  int32_t s = 0;
  for (int j = 0; j < 3; ++j) {
    uint64_t h = mix64(key + 3ull * index + (uint64_t)j);
    s += (int32_t)(h & 0xffff) + (int32_t)((h >> 16) & 0xffff) +
         (int32_t)((h >> 32) & 0xffff) + (int32_t)(h >> 48);
  }
  return fmul((float)(s - 393210), 1.0f / 65536.0f);
}

// fp16 bits -> fp32 (exact widening).
MLB_HD float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
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
  return bitsf(bits);
}

// fp32 -> fp16 bits with the reference's half-up rounding of the dropped bits.
MLB_HD uint16_t float_to_half_ref(float f) {
  uint32_t b = fbits(f);
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

MLB_HD int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Quantise n <= 32 values into one block; `out` receives 34/18/20 bytes.
MLB_HD void quantize_q8_0(const float* x, int n, uint8_t* out) {
  for (int i = 0; i < 34; ++i) out[i] = 0;
  float amax = 0.0f;
  for (int i = 0; i < n; ++i) {
    float a = fabs_(x[i]);
    if (a > amax) amax = a;
  }
  if (!(amax > 0.0f)) return;
  uint16_t d = float_to_half_ref(fdiv(amax, 127.0f));
  out[0] = (uint8_t)(d & 0xff);
  out[1] = (uint8_t)(d >> 8);
  float sd = half_to_float(d);
  float inv = sd == 0.0f ? 0.0f : fdiv(1.0f, sd);
  for (int i = 0; i < n; ++i)
    out[2 + i] = (uint8_t)(int8_t)clampi((int)fround(fmul(x[i], inv)), -127, 127);
}

MLB_HD void quantize_q4_0(const float* x, int n, uint8_t* out) {
  for (int i = 0; i < 18; ++i) out[i] = 0;
  float amax = 0.0f;
  for (int i = 0; i < n; ++i) {
    float a = fabs_(x[i]);
    if (a > amax) amax = a;
  }
  if (!(amax > 0.0f)) return;
  uint16_t d = float_to_half_ref(fdiv(amax, 7.0f));
  out[0] = (uint8_t)(d & 0xff);
  out[1] = (uint8_t)(d >> 8);
  float sd = half_to_float(d);
  float inv = sd == 0.0f ? 0.0f : fdiv(1.0f, sd);
  for (int j = 0; j < 16; ++j) {
    float v0 = j < n ? fmul(x[j], inv) : 0.0f;
    float v1 = j + 16 < n ? fmul(x[j + 16], inv) : 0.0f;
    int q0 = clampi((int)fround(fadd(v0, 8.0f)), 0, 15);
    int q1 = clampi((int)fround(fadd(v1, 8.0f)), 0, 15);
    out[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

MLB_HD void quantize_q4_1(const float* x, int n, uint8_t* out) {
  for (int i = 0; i < 20; ++i) out[i] = 0;
  float lo = bitsf(0x7f800000u), hi = bitsf(0xff800000u);
  for (int i = 0; i < n; ++i) {
    if (x[i] < lo) lo = x[i];
    if (x[i] > hi) hi = x[i];
  }
  float range = fsub(hi, lo);
  if (range > 0.0f) {
    uint16_t d = float_to_half_ref(fdiv(range, 15.0f));
    uint16_t m = float_to_half_ref(lo);
    out[0] = (uint8_t)(d & 0xff);
    out[1] = (uint8_t)(d >> 8);
    out[2] = (uint8_t)(m & 0xff);
    out[3] = (uint8_t)(m >> 8);
    float sd = half_to_float(d), sm = half_to_float(m);
    float inv = sd == 0.0f ? 0.0f : fdiv(1.0f, sd);
    for (int j = 0; j < 16; ++j) {
      int q0 = j < n ? clampi((int)fround(fmul(fsub(x[j], sm), inv)), 0, 15) : 0;
      int q1 = j + 16 < n ? clampi((int)fround(fmul(fsub(x[j + 16], sm), inv)), 0, 15) : 0;
      out[4 + j] = (uint8_t)(q0 | (q1 << 4));
    }
  } else {
    uint16_t m = float_to_half_ref(lo == bitsf(0x7f800000u) ? 0.0f : lo);
    out[2] = (uint8_t)(m & 0xff);
    out[3] = (uint8_t)(m >> 8);
  }
}

MLB_HD int block_bytes(int qtype) {
  return qtype == 1 ? 34 : (qtype == 2 ? 18 : (qtype == 3 ? 20 : 4));
}

// Writes block `b` of row `r` of a [*, cols] tensor (global indices) whose
// fp32 values are gauss(key, index) * scale.
MLB_HD void synth_block(int qtype, uint64_t key, float scale, int64_t r, int64_t b,
                        int64_t cols, uint8_t* out) {
  float v[32];
  int n = (int)(cols - b * 32 < 32 ? cols - b * 32 : 32);
  for (int i = 0; i < n; ++i)
    v[i] = fmul(gauss(key, (uint64_t)(r * cols + b * 32 + i)), scale);
  if (qtype == 1) quantize_q8_0(v, n, out);
  else if (qtype == 2) quantize_q4_0(v, n, out);
  else quantize_q4_1(v, n, out);
}

// Raw random blocks for the standalone GEMV sweep: fp16 scale |N(0,1)|*0.01,
// Q4_1 min N(0,1)*0.01, nibbles / int8 values uniform (Q8_0 in [-127, 127]).
MLB_HD void raw_block(int qtype, uint64_t key, uint64_t block_index, uint8_t* out) {
  uint64_t h0 = mix64(key + 5ull * block_index);
  float g0 = gauss(key ^ 0x5851F42D4C957F2Dull, block_index);
  uint16_t d = float_to_half_ref(fmul(fabs_(g0), 0.01f));
  out[0] = (uint8_t)(d & 0xff);
  out[1] = (uint8_t)(d >> 8);
  int off = 2;
  if (qtype == 3) {
    float g1 = gauss(key ^ 0x2545F4914F6CDD1Dull, block_index);
    uint16_t m = float_to_half_ref(fmul(g1, 0.01f));
    out[2] = (uint8_t)(m & 0xff);
    out[3] = (uint8_t)(m >> 8);
    off = 4;
  }
  if (qtype == 1) {
    for (int i = 0; i < 32; ++i) {
      uint64_t h = mix64(h0 + (uint64_t)i);
      out[2 + i] = (uint8_t)(int8_t)((int)(h % 255ull) - 127);
    }
  } else {
    for (int w = 0; w < 2; ++w) {
      uint64_t h = mix64(h0 + 100ull + (uint64_t)w);
      for (int i = 0; i < 8; ++i) out[off + w * 8 + i] = (uint8_t)(h >> (8 * i));
    }
  }
}

}  // namespace synth
}  // namespace mlb

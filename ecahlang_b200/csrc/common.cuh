// Device helpers shared by the sampler kernels: dtype traits, order-preserving
// keys, Philox4x32-10, and the exp used for softmax masses.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/ecah_sampler.h"

namespace ecah {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr float kLog2e = 1.4426950408889634f;
// Masses exp(z - M) below 2^-126 flush to zero in ex2.approx.ftz; every token
// with z < M - kExpCut has mass exactly 0 and is skipped without computing it.
constexpr float kExpCut = 96.0f;

// ------------------------------------------------------------------ dtypes
// Raw: the storage word of one logit.  to_f32 is exact; round() rounds a
// float32 to the model dtype (round-to-nearest-even), as torch does when it
// writes the result of an fp16/bf16 op computed in float32.
template <int DT> struct DType;

template <> struct DType<ECAH_DTYPE_F16> {
  using Raw = uint16_t;
  static constexpr int kVec = 8;  // logits per 16-byte load
  static __device__ __forceinline__ float to_f32(uint32_t r) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(r)));
  }
  static __device__ __forceinline__ float round(float f) { return __half2float(__float2half_rn(f)); }
  static __device__ __forceinline__ float round_down(float f) { return __half2float(__float2half_rd(f)); }
  static __device__ __forceinline__ uint32_t to_raw(float f) { return __half_as_ushort(__float2half_rn(f)); }
};

template <> struct DType<ECAH_DTYPE_BF16> {
  using Raw = uint16_t;
  static constexpr int kVec = 8;
  static __device__ __forceinline__ float to_f32(uint32_t r) { return __uint_as_float(r << 16); }
  static __device__ __forceinline__ float round(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
  static __device__ __forceinline__ float round_down(float f) { return __bfloat162float(__float2bfloat16_rd(f)); }
  static __device__ __forceinline__ uint32_t to_raw(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
};

template <> struct DType<ECAH_DTYPE_F32> {
  using Raw = uint32_t;
  static constexpr int kVec = 4;
  static __device__ __forceinline__ float to_f32(uint32_t r) { return __uint_as_float(r); }
  static __device__ __forceinline__ float round(float f) { return f; }
  static __device__ __forceinline__ float round_down(float f) { return f; }
  static __device__ __forceinline__ uint32_t to_raw(float f) { return __float_as_uint(f); }
};

// ------------------------------------------------------------------- keys
// Order-preserving unsigned keys: key(a) < key(b) iff a < b for non-NaN
// values (-0 sorts just below +0).  16-bit keys are built from the fp16/bf16
// bit pattern itself (a logit that stays in the model dtype), 32-bit keys
// from the float32 value (fp32 logits or additive penalties).
__device__ __forceinline__ uint32_t key16(uint32_t r) { return r ^ ((r & 0x8000u) ? 0xFFFFu : 0x8000u); }
__device__ __forceinline__ uint32_t unkey16(uint32_t k) { return k ^ ((k & 0x8000u) ? 0x8000u : 0xFFFFu); }
// two packed 16-bit raws -> two packed keys
__device__ __forceinline__ uint32_t key16x2(uint32_t w) {
  uint32_t neg = (w >> 15) & 0x00010001u;
  return w ^ ((neg * 0x7FFFu) | 0x80008000u);
}
__device__ __forceinline__ uint32_t key32(float f) {
  uint32_t b = __float_as_uint(f);
  return b ^ (static_cast<uint32_t>(static_cast<int32_t>(b) >> 31) | 0x80000000u);
}
__device__ __forceinline__ float unkey32(uint32_t k) {
  return __uint_as_float(k ^ (static_cast<uint32_t>(static_cast<int32_t>(~k) >> 31) | 0x80000000u));
}

// Codec<DT, KB>: key type and conversions for KB-bit keys of dtype DT.
template <int DT, int KB> struct Codec;

template <int DT> struct Codec<DT, 16> {
  using Key = uint16_t;
  static constexpr int kBits = 16;
  static __device__ __forceinline__ uint32_t from_raw(uint32_t r) { return key16(r); }
  // v must already be a value of the model dtype
  static __device__ __forceinline__ uint32_t from_val(float v) { return key16(DType<DT>::to_raw(v)); }
  static __device__ __forceinline__ float value(uint32_t k) { return DType<DT>::to_f32(unkey16(k)); }
};

template <int DT> struct Codec<DT, 32> {
  using Key = uint32_t;
  static constexpr int kBits = 32;
  static __device__ __forceinline__ uint32_t from_raw(uint32_t r) { return key32(DType<DT>::to_f32(r)); }
  static __device__ __forceinline__ uint32_t from_val(float v) { return key32(v); }
  static __device__ __forceinline__ float value(uint32_t k) { return unkey32(k); }
};

// --------------------------------------------------------------- Philox
// Philox4x32-10 (Salmon et al., SC'11), written from the paper.
struct U4 { uint32_t x, y, z, w; };

__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) { k0 += W0; k1 += W1; }
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
  }
  return c;
}

// Uniform in [0,1) for one row: counter = (row, offset), key = seed.
__device__ __forceinline__ float row_uniform(uint64_t seed, uint64_t offset, uint64_t row) {
  U4 c{static_cast<uint32_t>(row), static_cast<uint32_t>(row >> 32), static_cast<uint32_t>(offset),
       static_cast<uint32_t>(offset >> 32)};
  U4 o = philox4x32_10(c, static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  return static_cast<float>(o.x >> 8) * 5.9604644775390625e-08f;  // 2^-24
}

// -------------------------------------------------------------- numerics
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// y / T from the reciprocal rT = __frcp_rn(T) with one correction step
// (Markstein, "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990): q = RN(y rT), r = RN(y - q T)
// (exact through the fma), q' = RN(q + r rT).  ecah_quotient_mismatches
// compares it with the IEEE quotient over every fp16 and bf16 input and over
// every float32 input, per temperature.
__device__ __forceinline__ float quot_rn(float y, float T, float rT) {
  const float q = __fmul_rn(y, rT);
  return __fmaf_rn(__fmaf_rn(-q, T, y), rT, q);
}

// Unnormalised softmax mass of a token whose (penalised) logit is y:
// z = y / T rounded to float32 exactly as torch's divide, then exp(z - M).
__device__ __forceinline__ float token_mass(float y, float T, float M) {
  const float z = __fdiv_rn(y, T);
  return ex2_approx(__fmul_rn(__fsub_rn(z, M), kLog2e));
}

// Mask value after `count` updates of the reference rule
// (m /= rp if rp > 1 else m *= rp, in the model dtype).  torch applies both to
// a CUDA tensor as one float32 multiply by `factor` = float32(1/rp) (reciprocal
// in double) or float32(rp), then rounds to the model dtype; the host passes
// that factor.
// The loop stops at a fixed point (m unchanged, e.g. rp == 1 or m == 0) or a
// NaN, and never runs more than kMaxPenaltySteps times (only a negative
// factor, which the request layer cannot produce, reaches that cap).
constexpr int kMaxPenaltySteps = 1 << 16;

template <int DT>
__device__ __forceinline__ float penalty_divisor(int count, float f) {
  float m = 1.0f;
  const int steps = min(count, kMaxPenaltySteps);
  for (int i = 0; i < steps; ++i) {
    const float next = DType<DT>::round(__fmul_rn(m, f));
    if (next == m || next != next) { m = next; break; }
    m = next;
  }
  return m;
}

template <int DT>
__device__ __forceinline__ float penalty_step(float m, float factor) {
  return DType<DT>::round(__fmul_rn(m, factor));
}

}  // namespace ecah

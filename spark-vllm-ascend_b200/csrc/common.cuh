// common.cuh -- shared device helpers for the Spark B200 decode kernels (sm_100a only).
//
// Numerics contract: every kernel evaluates the canonical fp32 order that the CPU
// oracle restates (oracle/spark_oracle.c), so results are bit-identical.  The
// device exp/log below are this project's own implementation (Cody-Waite range
// reduction with a degree-7 Taylor polynomial; log through the atanh series),
// written with plain IEEE fp32 operations so that the host restatement reproduces
// them exactly.  No fast-math: the library is compiled without -use_fast_math so
// every division and square root is IEEE round-to-nearest.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "spark_b200 kernels target sm_100a (B200) only"
#endif

namespace spark {

constexpr int kNumSMs = 148;

// ---------------------------------------------------------------- status codes
enum Status : int {
  kOk = 0,
  kErrInvalidArg = 1,
  kErrUnsupportedShape = 2,
  kErrAlignment = 3,
  kErrLaunch = 4,
  kErrTooLarge = 5,
};

// ---------------------------------------------------------------- bf16 / fp32
__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

// round-to-nearest-even; NaN -> 0x7fff (same rule as the host restatement)
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fff;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---------------------------------------------------------------- exp / log
constexpr float kLog2e = 1.44269502162933349609375f;  // fp32(log2 e)
constexpr float kLn2Hi = 0.693145751953125f;          // ln 2 to 16 significant bits
constexpr float kLn2Lo = 1.428606765330187e-06f;      // ln 2 - kLn2Hi

__device__ __forceinline__ float spark_exp(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return __int_as_float(0x7f800000);
  if (x < -104.0f) return 0.0f;
  float n = rintf(__fmul_rn(x, kLog2e));
  float r = __fmaf_rn(-n, kLn2Hi, x);
  r = __fmaf_rn(-n, kLn2Lo, r);
  float p = 1.98412698e-04f;
  p = __fmaf_rn(p, r, 1.38888889e-03f);
  p = __fmaf_rn(p, r, 8.33333377e-03f);
  p = __fmaf_rn(p, r, 4.16666679e-02f);
  p = __fmaf_rn(p, r, 1.66666672e-01f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ni = (int)n;
  if (ni >= -126 && ni <= 127) return __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
  int n1 = ni / 2, n2 = ni - n1;
  return __fmul_rn(__fmul_rn(p, __uint_as_float((uint32_t)(n1 + 127) << 23)),
                   __uint_as_float((uint32_t)(n2 + 127) << 23));
}

// spark_exp for x <= 0 (or -inf) without branches: the same reduction and polynomial,
// and the scaling by 2^n always as two exact steps (p 2^(n/2)) 2^(n - n/2), which rounds
// once, where spark_exp rounds once in p 2^n: bit-identical to spark_exp on x <= 0.
// Arguments below -104 give 0 (spark_exp's cut); NaN is not expected.
__device__ __forceinline__ float spark_exp_neg(float x) {
  const float n = rintf(__fmul_rn(x, kLog2e));
  float r = __fmaf_rn(-n, kLn2Hi, x);
  r = __fmaf_rn(-n, kLn2Lo, r);
  float p = 1.98412698e-04f;
  p = __fmaf_rn(p, r, 1.38888889e-03f);
  p = __fmaf_rn(p, r, 8.33333377e-03f);
  p = __fmaf_rn(p, r, 4.16666679e-02f);
  p = __fmaf_rn(p, r, 1.66666672e-01f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = x < -104.0f ? 0 : (int)n;  // (the result is discarded below -104)
  const int n1 = ni / 2, n2 = ni - n1;
  const float v = __fmul_rn(__fmul_rn(p, __uint_as_float((uint32_t)(n1 + 127) << 23)),
                            __uint_as_float((uint32_t)(n2 + 127) << 23));
  return x < -104.0f ? 0.0f : v;
}

// GELU of a bf16 value as the reference's activation table (kernels/linear.py:540-577,
// table built in integration/model.py:12-16): table [4096] = gelu of the bf16 inputs
// 0x3b00 + i and 0xbb00 + i (|x| in [2^-9, 128)); |x| < 2^-9: bf16(x / 2); x >= 128: x;
// x <= -128: -0; NaN and -inf: 0x7fff.
__device__ __forceinline__ uint16_t spark_gelu_bf16(uint16_t x, const uint16_t* table) {
  const uint32_t ab = x & 0x7fffu;
  if (ab > 0x7f80u || x == 0xff80u) return 0x7fff;
  if (x >= 0xc300u) return 0x8000;
  if (ab >= 0x4300u) return x;
  if (ab < 0x3b00u) return f2bf(__fmul_rn(0.5f, bf2f(x)));
  return __ldg(table + ((ab - 0x3b00u) | ((uint32_t)(x >> 4) & 0x800u)));
}

__device__ __forceinline__ float spark_log(float x) {
  if (x != x || x < 0.0f) return __int_as_float(0x7fc00000);
  if (x == 0.0f) return __int_as_float(0xff800000);
  if (x == __int_as_float(0x7f800000)) return x;
  uint32_t u = __float_as_uint(x);
  int e = (int)(u >> 23) - 127;
  if ((u >> 23) == 0) {
    x = __fmul_rn(x, 8388608.0f);
    u = __float_as_uint(x);
    e = (int)(u >> 23) - 127 - 23;
  }
  float m = __uint_as_float((u & 0x7fffffu) | 0x3f800000u);
  if (m > 1.41421354f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  float f = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  float f2 = __fmul_rn(f, f);
  float s = 9.09090936e-02f;
  s = __fmaf_rn(s, f2, 1.11111112e-01f);
  s = __fmaf_rn(s, f2, 1.42857149e-01f);
  s = __fmaf_rn(s, f2, 2.00000003e-01f);
  s = __fmaf_rn(s, f2, 3.33333343e-01f);
  s = __fmaf_rn(s, f2, 1.0f);
  float lm = __fmul_rn(__fmul_rn(2.0f, f), s);
  float fe = (float)e;
  return __fmaf_rn(fe, kLn2Hi, __fmaf_rn(fe, kLn2Lo, lm));
}

// ---------------------------------------------------------------- warp helpers
template <int kWidth>
__device__ __forceinline__ float butterfly_sum(float v) {
#pragma unroll
  for (int off = kWidth / 2; off >= 1; off /= 2) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off /= 2) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// ---------------------------------------------------------------- programmatic dependent launch
// Wait for the preceding kernel in the stream (no-op when launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next kernel in the stream to start its prologue.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------- memory helpers
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ldg_u16_stream(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

}  // namespace spark

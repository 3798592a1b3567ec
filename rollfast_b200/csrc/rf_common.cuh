// Shared device/host helpers for the rollfast_b200 kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/rollfast_b200.h"

namespace rf {

// ---------------------------------------------------------------------------
// Host-side error plumbing: every entry point returns an rf_status and keeps
// a thread-local message for rf_last_error().
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
rf_status fail(rf_status st, const std::string& msg);
rf_status check_launch(const char* what);
void count_launch(int n = 1);

#define RF_TRY(expr)                     \
  do {                                   \
    rf_status _st = (expr);              \
    if (_st != RF_OK) return _st;        \
  } while (0)

// Device-side error word (library static, one per device that loads the
// library).  Bounded waits that give up set it; rf_muon_update and friends
// report it through rf_device_error() (see rf_api.cu).
enum DeviceError : int { kDevOk = 0, kDevTimeoutProducer = 1, kDevTimeoutMma = 2, kDevTimeoutEpilogue = 3 };

// ---------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ld_as_float(const void* p, int dt, int64_t i) {
  if (dt == RF_F32) return static_cast<const float*>(p)[i];
  if (dt == RF_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void st_from_float(void* p, int dt, int64_t i, float v) {
  if (dt == RF_F32) {
    static_cast<float*>(p)[i] = v;
  } else if (dt == RF_BF16) {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

// Round a float to the given storage dtype and back (the value a 16-bit
// array would hold).
__device__ __forceinline__ float round_to(int dt, float v) {
  if (dt == RF_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == RF_F16) return __half2float(__float2half_rn(v));
  return v;
}

// Optax add_decayed_weights forms `weight_decay * p` with a weakly typed
// Python float, i.e. in the parameter dtype (`decay` arrives already rounded
// to that dtype by the host); a strongly typed float32 weight decay (a
// schedule's array value, or the in-transform decay of scale_by_adam) forms
// it in float32 (rdt = RF_F32).
__device__ __forceinline__ float decay_term(int rdt, float decay, float p) {
  return round_to(rdt, decay * p);
}

// Stochastic rounding to bfloat16 (utils.py:342-371): 16 bits of noise added
// below the bf16 significand, then truncation; +-Inf / NaN get no noise.  The
// noise is the SplitMix64 sequence (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", 2014) of a per-leaf seed: output c serves
// elements 4c..4c+3, 16 bits each from the low end.
__device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t c) {
  uint64_t z = seed + (c + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float sr_bf16(float x, uint32_t noise16) {
  uint32_t b = __float_as_uint(x);
  if ((b & 0x7FFFFFFFu) >= 0x7F800000u) noise16 = 0u;
  return __uint_as_float((b + noise16) & 0xFFFF0000u);
}

__device__ __forceinline__ uint32_t sr_noise(uint64_t seed, int64_t i) {
  return uint32_t((splitmix64_at(seed, uint64_t(i) >> 2) >> (16 * (i & 3))) & 0xFFFFu);
}

// A float32 value stored to `dt` at p[i]: bfloat16 with stochastic rounding
// when `sr` (noise of element i of the seed's stream), else nearest-even.
__device__ __forceinline__ void st_rounded(void* p, int dt, int64_t i, float v, bool sr, uint64_t seed) {
  if (sr && dt == RF_BF16) {
    static_cast<uint16_t*>(p)[i] = uint16_t(__float_as_uint(sr_bf16(v, sr_noise(seed, i))) >> 16);
  } else {
    st_from_float(p, dt, i, v);
  }
}

inline size_t dtype_size(int dt) { return dt == RF_F32 ? 4 : 2; }
inline bool valid_dtype(int dt) { return dt == RF_F32 || dt == RF_BF16 || dt == RF_F16; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }
inline size_t align_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

// ---------------------------------------------------------------------------
// Newton-Schulz operand scaling.  16-bit operands are stored pre-multiplied
// by powers of two so that float16 keeps its 11-bit significand over the
// whole iteration (entries of X, A = XX^T and B = bA + cA^2 shrink like
// 1/sqrt(m), 1/m early on).  Power-of-two scales are exact, so they change
// no value; they are folded into the epilogue coefficients.
// ---------------------------------------------------------------------------
struct NsScales {
  float sx, sa, sb;
};
inline NsScales ns_scales(int64_t m, int precision) {
  NsScales s{1.f, 1.f, 1.f};
  if (precision == RF_NS_F32) return s;
  int lg = 0;
  while ((int64_t(1) << (lg + 1)) <= m) ++lg;  // floor(log2 m)
  s.sx = float(1 << ((lg + 1) / 2));            // ~sqrt(m)
  s.sa = float(int64_t(1) << lg);               // <= m
  s.sb = s.sa / 8.f;
  if (s.sb < 1.f) s.sb = 1.f;
  return s;
}

}  // namespace rf

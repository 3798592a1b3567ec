// HBM-bound kernels of the Muon step (sm_100a):
//   k_momentum_sumsq   momentum update + Nesterov/bias-corrected direction,
//                      per-chunk partial sums of direction^2     (utils.py:437-645)
//   k_norm_finalize    per-matrix 1/(||d||_F + eps) from the partials
//                      (orthogonalization.py:243-246)
//   k_ns_load          direction -> scaled 16-bit (or fp32) NS operand, tiled
//                      transpose for rows > cols, zero padding (orthogonalization.py:227-231)
//   k_adamw            (N)AdamW fallback leaves (adam.py:123-177) + decay + LR
//   k_tail             -lr * (shape_scale * O + decay * p)  (muon.py:79-139, 390-393, 466)
//
// All leaf tables travel as kernel parameters (large-parameter launches), so
// every launch is self-contained and capturable in a CUDA graph.
#include "rf_kernels.cuh"

namespace rf {

// ---------------------------------------------------------------------------
// Direction formula (the reference's _prepare_first_moment_runtime with
// bias_correction=True, nesterov_moment_count_offset=1).  All products and
// sums are rounded separately (no FMA contraction) so `mu` matches the
// reference's float32 arithmetic bit for bit.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float momentum_new(const MomentumCoeffs& c, float g, float mu) {
  return __fadd_rn(__fmul_rn(c.s, g), __fmul_rn(c.beta, mu));
}

__device__ __forceinline__ float direction(const MomentumCoeffs& c, float g, float mu_new) {
  switch (c.mode) {
    case kDirEmaNesterov:
      return __fadd_rn(__fmul_rn(c.beta, __fdiv_rn(mu_new, c.bc_mu)),
                       __fmul_rn(c.s, __fdiv_rn(g, c.bc_g)));
    case kDirEma:
      return __fdiv_rn(mu_new, c.bc_mu);
    case kDirHeavyBallNesterov:
      return __fadd_rn(__fmul_rn(c.beta, mu_new), __fmul_rn(c.s, g));
    case kDirHeavyBall:
      return mu_new;
    default:  // kDirIdentity: plain NS input (orthogonalize_fn seam)
      return g;
  }
}

// The same direction with reciprocal multiplies instead of IEEE divisions:
// used only where the result is immediately rounded to the 16-bit (or
// scaled float32) Newton-Schulz operand, so the last-bit difference never
// reaches the momentum state.
__device__ __forceinline__ float direction_fast(const MomentumCoeffs& c, float g, float mu_new) {
  switch (c.mode) {
    case kDirEmaNesterov:
      return fmaf(c.beta * c.rbc_mu, mu_new, c.s * c.rbc_g * g);
    case kDirEma:
      return mu_new * c.rbc_mu;
    case kDirHeavyBallNesterov:
      return fmaf(c.beta, mu_new, c.s * g);
    case kDirHeavyBall:
      return mu_new;
    default:
      return g;
  }
}

template <int GDT>
struct GradVec;
template <>
struct GradVec<RF_F32> {
  static __device__ __forceinline__ void load8(const void* p, int64_t i, float* v) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    float4 a = __ldcs(q), b = __ldcs(q + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};
template <>
struct GradVec<RF_BF16> {
  static __device__ __forceinline__ void load8(const void* p, int64_t i, float* v) {
    uint4 raw = __ldcs(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + i));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = __bfloat1622float2(h[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
  }
};
template <>
struct GradVec<RF_F16> {
  static __device__ __forceinline__ void load8(const void* p, int64_t i, float* v) {
    uint4 raw = __ldcs(reinterpret_cast<const uint4*>(static_cast<const __half*>(p) + i));
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = __half22float2(h[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
  }
};

__device__ __forceinline__ int find_leaf(const int64_t* begins, int n, int64_t key) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (begins[mid] <= key) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = (l < int(blockDim.x >> 5)) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in thread 0
}

// ---------------------------------------------------------------------------
// Stochastic rounding to bfloat16 (utils.py:342-371): 16 bits of noise added
// below the bf16 significand, then truncation; +-Inf / NaN get no noise.
// The noise is the SplitMix64 sequence (Steele, Lea and Flood, "Fast
// splittable pseudorandom number generators", 2014) of a per-leaf seed:
// output c serves elements 4c..4c+3, 16 bits each from the low end.  Used for
// bfloat16 optimizer state (utils.py:412-425, adam.py:219-222) and
// apply_updates.
// ---------------------------------------------------------------------------
// v[0..7] -> bf16 at p[i..i+7] (i % 8 == 0, 16-byte aligned), stochastically rounded.
__device__ __forceinline__ void sr_store8_bf16(void* p, int64_t i, const float* v, uint64_t seed) {
  const uint64_t r0 = splitmix64_at(seed, uint64_t(i) >> 2), r1 = splitmix64_at(seed, (uint64_t(i) >> 2) + 1);
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = __float_as_uint(sr_bf16(v[2 * k], uint32_t(((k < 2 ? r0 : r1) >> (32 * (k & 1))) & 0xFFFFu)));
    const uint32_t hi =
        __float_as_uint(sr_bf16(v[2 * k + 1], uint32_t(((k < 2 ? r0 : r1) >> (32 * (k & 1) + 16)) & 0xFFFFu)));
    w[k] = (lo >> 16) | (hi & 0xFFFF0000u);
  }
  *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p) + i) = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void sr_store1_bf16(void* p, int64_t i, float v, uint64_t seed) {
  static_cast<uint16_t*>(p)[i] = uint16_t(__float_as_uint(sr_bf16(v, sr_noise(seed, i))) >> 16);
}

__device__ __forceinline__ float ld_bf16(const void* p, int64_t i) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

// ---------------------------------------------------------------------------
// k_momentum_sumsq: one CTA per chunk of kChunk elements of one matrix.
// ---------------------------------------------------------------------------
template <int GDT>
__global__ void __launch_bounds__(kEwThreads) k_momentum_sumsq(const __grid_constant__ MomentumLaunch P) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  __shared__ float red[32];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].chunk_begin;
  __syncthreads();
  for (int64_t chunk = blockIdx.x; chunk < P.total_chunks; chunk += gridDim.x) {
    const int li = find_leaf(s_begin, P.n, chunk);
    const MomentumLeaf& L = P.leaf[li];
    const int64_t local = chunk - L.chunk_begin;
    const int64_t mat = local / L.chunks_per_mat;
    const int64_t cim = local - mat * L.chunks_per_mat;
    const int64_t base = mat * L.numel;
    const int64_t lo = cim * kChunk;
    const int64_t hi = (lo + kChunk < L.numel ? lo + kChunk : L.numel);
    float acc = 0.f;
    if (L.vec_ok && L.mu_bf16) {
      // bfloat16 state: the new momentum only feeds the norm here; the
      // operand load recomputes it and stores it (stochastically rounded).
      for (int64_t i = lo + int64_t(threadIdx.x) * 8; i < hi; i += int64_t(blockDim.x) * 8) {
        float g[8], m[8];
        GradVec<GDT>::load8(L.g, base + i, g);
        GradVec<RF_BF16>::load8(L.mu, base + i, m);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          m[k] = momentum_new(P.c, g[k], m[k]);
          const float d = direction(P.c, g[k], m[k]);
          acc = fmaf(d, d, acc);
        }
      }
    } else if (L.vec_ok && !L.mu) {
      // No momentum (the orthogonalize_fn seam): sum of squares of the input.
      for (int64_t i = lo + int64_t(threadIdx.x) * 8; i < hi; i += int64_t(blockDim.x) * 8) {
        float g[8];
        GradVec<GDT>::load8(L.g, base + i, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float d = direction(P.c, g[k], 0.f);
          acc = fmaf(d, d, acc);
        }
      }
    } else if (L.vec_ok) {
      for (int64_t i = lo + int64_t(threadIdx.x) * 8; i < hi; i += int64_t(blockDim.x) * 8) {
        float g[8], m[8];
        GradVec<GDT>::load8(L.g, base + i, g);
        float4* mp = reinterpret_cast<float4*>(L.mu + base + i);
        float4 m0 = mp[0], m1 = mp[1];
        m[0] = m0.x; m[1] = m0.y; m[2] = m0.z; m[3] = m0.w;
        m[4] = m1.x; m[5] = m1.y; m[6] = m1.z; m[7] = m1.w;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          m[k] = momentum_new(P.c, g[k], m[k]);
          const float d = direction(P.c, g[k], m[k]);
          acc = fmaf(d, d, acc);
        }
        mp[0] = make_float4(m[0], m[1], m[2], m[3]);
        mp[1] = make_float4(m[4], m[5], m[6], m[7]);
      }
    } else {
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float g = ld_as_float(L.g, GDT, base + i);
        float m = L.mu ? (L.mu_bf16 ? ld_bf16(L.mu, base + i) : L.mu[base + i]) : 0.f;
        if (L.mu) {
          m = momentum_new(P.c, g, m);
          if (!L.mu_bf16) L.mu[base + i] = m;
        }
        const float d = direction(P.c, g, m);
        acc = fmaf(d, d, acc);
      }
    }
    const float t = block_sum(acc, red);
    if (threadIdx.x == 0) P.partials[chunk] = t;
  }
}

// Plain sum of squares (orthogonalize_fn seam, no momentum): same kernel with
// mu == nullptr and kDirIdentity.

// ---------------------------------------------------------------------------
// k_norm_finalize: one CTA per matrix, fixed-order reduction of its partials.
// denom[mat] = ||d||_F + eps (orthogonalization.py:244-246).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEwThreads) k_norm_finalize(const __grid_constant__ MomentumLaunch P,
                                                              float* __restrict__ denom_out, float eps) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  __shared__ float red[32];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].mat_begin;
  __syncthreads();
  for (int64_t mat = blockIdx.x; mat < P.total_mats; mat += gridDim.x) {
    const int li = find_leaf(s_begin, P.n, mat);
    const MomentumLeaf& L = P.leaf[li];
    const int64_t local_mat = mat - L.mat_begin;
    const int64_t c0 = L.chunk_begin + local_mat * L.chunks_per_mat;
    float acc = 0.f;
    for (int64_t i = threadIdx.x; i < L.chunks_per_mat; i += blockDim.x) acc += P.partials[c0 + i];
    const float t = block_sum(acc, red);
    if (threadIdx.x == 0) {
      denom_out[L.scale_index + local_mat] = __fadd_rn(__fsqrt_rn(t), eps);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// k_ns_load: builds the padded NS operand X~0 = round(d * (sx / (||d|| + eps)))
// for every matrix of one shape group, 64x64 output tiles.  Each thread
// moves 8-element vectors (16-byte grad / operand accesses, 32-byte mu).
// A leaf with rows <= cols maps straight onto the operand; a transposed leaf
// (rows > cols) is staged through shared memory so that both the leaf rows
// and the operand rows are read and written contiguously.
// ---------------------------------------------------------------------------
template <int GDT>
__device__ __forceinline__ void load8_any(const void* p, int64_t i, float* v) {
  GradVec<GDT>::load8(p, i, v);
}

template <typename OT>
__device__ __forceinline__ void store8(OT* p, const float* v);
template <>
__device__ __forceinline__ void store8<float>(float* p, const float* v) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float* v) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// 8 consecutive scaled directions of leaf row `ir`, columns ic..ic+7 (zero
// outside the leaf).
template <int GDT>
__device__ __forceinline__ void dir8(const LoadLaunch& P, const LoadLeaf& L, int64_t base, int64_t ir, int64_t ic,
                                     float scale, float* v) {
  if (ir < L.rows && ic + 7 < L.cols && L.vec_ok) {
    const int64_t idx = base + ir * L.cols + ic;
    float g[8], m[8];
    load8_any<GDT>(L.g, idx, g);
    if (L.mu && L.mu_bf16) {
      GradVec<RF_BF16>::load8(L.mu, idx, m);
#pragma unroll
      for (int k = 0; k < 8; ++k) m[k] = momentum_new(P.c, g[k], m[k]);
      if (L.store_mu) sr_store8_bf16(const_cast<float*>(L.mu), idx, m, L.sr_seed);
    } else if (L.mu) {
      const float4* mp = reinterpret_cast<const float4*>(L.mu + idx);
      const float4 a = mp[0], b = mp[1];
      m[0] = a.x; m[1] = a.y; m[2] = a.z; m[3] = a.w; m[4] = b.x; m[5] = b.y; m[6] = b.z; m[7] = b.w;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) m[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = direction_fast(P.c, g[k], m[k]) * scale;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t c = ic + k;
      float x = 0.f;
      if (ir < L.rows && c < L.cols) {
        const int64_t idx = base + ir * L.cols + c;
        const float g = ld_as_float(L.g, GDT, idx);
        float m = 0.f;
        if (L.mu && L.mu_bf16) {
          m = momentum_new(P.c, g, ld_bf16(L.mu, idx));
          if (L.store_mu) sr_store1_bf16(const_cast<float*>(L.mu), idx, m, L.sr_seed);
        } else if (L.mu) {
          m = L.mu[idx];
        }
        x = direction_fast(P.c, g, m) * scale;
      }
      v[k] = x;
    }
  }
}

template <int GDT, typename OT>
__global__ void __launch_bounds__(256) k_ns_load(const __grid_constant__ LoadLaunch P) {
  __shared__ float tile[64][65];
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].group_mat_begin;
  __syncthreads();
  const int64_t tiles_c = P.np / 64;
  const int64_t tiles_per_mat = (P.mp / 64) * tiles_c;
  const int64_t total = tiles_per_mat * P.group_mats;
  const int tr = threadIdx.x >> 3;        // 0..31: tile row (and +32)
  const int tc = (threadIdx.x & 7) * 8;   // 0..56: 8-column group
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t gm = t / tiles_per_mat;
    const int64_t tl = t - gm * tiles_per_mat;
    const int64_t r0 = (tl / tiles_c) * 64, c0 = (tl % tiles_c) * 64;
    const LoadLeaf& L = P.leaf[find_leaf(s_begin, P.n, gm)];
    if (L.gdt != GDT) continue;  // uniform per tile: another launch covers it
    const int64_t bi = gm - L.group_mat_begin;
    const int64_t base = bi * L.rows * L.cols;
    // sx / (||d|| + eps): one division per tile; sx is a power of two.
    const float scale = P.sx / P.denom[L.norm_index + bi];
    OT* out = static_cast<OT*>(P.x) + gm * P.mp * P.np;
    const float* rs = P.row_scale ? P.row_scale + gm * P.mp : nullptr;
    if (!L.transposed) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t r = r0 + tr + 32 * h;
        float v[8];
        dir8<GDT>(P, L, base, r, c0 + tc, rs ? P.sx * rs[r] : scale, v);
        store8<OT>(out + r * P.np + c0 + tc, v);
      }
    } else {
      // Operand (r, c) = leaf (c, r): read leaf rows c0.., columns r0..
      __syncthreads();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int lr = tr + 32 * h;
        float v[8];
        dir8<GDT>(P, L, base, c0 + lr, r0 + tc, rs ? P.sx : scale, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) tile[lr][tc + k] = v[k];
      }
      __syncthreads();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int orow = tr + 32 * h;
        float v[8];
        // With row factors, sx (a power of two) was applied exactly above and
        // the factor rounds once here, as in the untransposed branch.
        const float f = rs ? rs[r0 + orow] : 1.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = rs ? tile[tc + k][orow] * f : tile[tc + k][orow];
        store8<OT>(out + (r0 + orow) * P.np + c0 + tc, v);
      }
    }
  }
}

// 8-element vector access with a runtime (warp-uniform) dtype.
__device__ __forceinline__ void ld8(const void* p, int dt, int64_t i, float* v) {
  if (dt == RF_F32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 a = q[0], b = q[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else if (dt == RF_BF16) {
    GradVec<RF_BF16>::load8(p, i, v);
  } else {
    GradVec<RF_F16>::load8(p, i, v);
  }
}
__device__ __forceinline__ void st8(void* p, int dt, int64_t i, const float* v) {
  if (dt == RF_F32) store8<float>(static_cast<float*>(p) + i, v);
  else if (dt == RF_BF16) store8<__nv_bfloat16>(static_cast<__nv_bfloat16*>(p) + i, v);
  else store8<__half>(static_cast<__half*>(p) + i, v);
}

__device__ __forceinline__ float adam_one(const AdamCoeffs& c, const AdamLeafDev& L, float g, float& mu, float& nu,
                                          float p, bool decay_on) {
  mu = __fadd_rn(__fmul_rn(c.one_minus_b1, g), __fmul_rn(c.b1, mu));
  nu = __fadd_rn(__fmul_rn(c.one_minus_b2, __fmul_rn(g, g)), __fmul_rn(c.b2, nu));
  float mh;
  if (c.nesterov) {
    mh = __fadd_rn(__fmul_rn(c.b1, __fdiv_rn(mu, c.bc1_next)), __fmul_rn(c.one_minus_b1_py, __fdiv_rn(g, c.bc1)));
  } else {
    mh = __fdiv_rn(mu, c.bc1);
  }
  const float nh = __fdiv_rn(nu, c.bc2);
  float u = __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(__fadd_rn(nh, c.eps_root)), c.eps));
  if (decay_on) u = __fadd_rn(u, decay_term(L.decay_dt, L.decay, p));
  if (L.scale_dev) u = __fmul_rn(*L.scale_dev, u);  // Magma: (keep * score) * u (magma.py:126-128)
  return __fmul_rn(c.neg_lr, u);
}

// ---------------------------------------------------------------------------
// k_adamw: multi-tensor (N)AdamW (8-element vectors where aligned).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEwThreads) k_adamw(const __grid_constant__ AdamLaunch P) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].chunk_begin;
  __syncthreads();
  const AdamCoeffs& c = P.c;
  for (int64_t chunk = blockIdx.x; chunk < P.total_chunks; chunk += gridDim.x) {
    const int li = find_leaf(s_begin, P.n, chunk);
    const AdamLeafDev& L = P.leaf[li];
    const int64_t lo = (chunk - L.chunk_begin) * kChunk;
    const int64_t hi = (lo + kChunk < L.n ? lo + kChunk : L.n);
    if (L.vec_ok) {
      for (int64_t i = lo + int64_t(threadIdx.x) * 8; i < hi; i += int64_t(blockDim.x) * 8) {
        float g[8], mu[8], nu[8], p[8], u[8];
        ld8(L.g, L.gdt, i, g);
        ld8(L.mu, L.sdt, i, mu);
        ld8(L.nu, L.sdt, i, nu);
        if (L.decay != 0.f || L.apply_mode) ld8(L.p, L.pdt, i, p);
        uint2 mk = make_uint2(0x01010101u, 0x01010101u);
        if (L.mask) mk = *reinterpret_cast<const uint2*>(L.mask + i);
        const uint8_t* mb = reinterpret_cast<const uint8_t*>(&mk);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          u[k] = adam_one(c, L, g[k], mu[k], nu[k], L.decay != 0.f ? p[k] : 0.f, L.decay != 0.f && mb[k] != 0);
        if (L.sdt == RF_BF16) {  // adam.py:219-222: both moments stochastically rounded
          sr_store8_bf16(L.mu, i, mu, L.seed_mu);
          sr_store8_bf16(L.nu, i, nu, L.seed_nu);
        } else {
          st8(L.mu, RF_F32, i, mu);
          st8(L.nu, RF_F32, i, nu);
        }
        if (L.apply_mode) {  // the new parameter p + u (utils.py:648-708)
#pragma unroll
          for (int k = 0; k < 8; ++k) u[k] = __fadd_rn(p[k], u[k]);
          if (L.apply_mode == 2 && L.odt == RF_BF16) {
            sr_store8_bf16(L.out, i, u, L.apply_seed);
            continue;
          }
        }
        st8(L.out, L.odt, i, u);
      }
    } else {
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float g = ld_as_float(L.g, L.gdt, i);
        float mu = ld_as_float(L.mu, L.sdt, i), nu = ld_as_float(L.nu, L.sdt, i);
        const float p = (L.decay != 0.f || L.apply_mode) ? ld_as_float(L.p, L.pdt, i) : 0.f;
        const float u = adam_one(c, L, g, mu, nu, p, L.decay != 0.f && (!L.mask || L.mask[i] != 0));
        if (L.sdt == RF_BF16) {
          sr_store1_bf16(L.mu, i, mu, L.seed_mu);
          sr_store1_bf16(L.nu, i, nu, L.seed_nu);
        } else {
          static_cast<float*>(L.mu)[i] = mu;
          static_cast<float*>(L.nu)[i] = nu;
        }
        if (L.apply_mode) st_rounded(L.out, L.odt, i, __fadd_rn(p, u), L.apply_mode == 2, L.apply_seed);
        else st_from_float(L.out, L.odt, i, u);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Magma (magma.py:86-128).  k_magma_dot: per chunk of one leaf, the sums
// <g, mu_t>, <g, g>, <mu_t, mu_t> in float32 with mu_t recomputed exactly as
// the momentum kernels form it.  k_magma_finalize: one CTA per leaf sums its
// chunks in a fixed order, then cos = clip(nan_to_num(dot / max(|g| |mu_t|,
// 1e-12)), -1, 1), score <- 0.9 score + 0.1 sigmoid(cos / tau), factor =
// keep * score (the leaf's Bernoulli draw times its new score).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEwThreads) k_magma_dot(const __grid_constant__ MagmaDotLaunch P) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  __shared__ float red[32];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].chunk_begin;
  __syncthreads();
  for (int64_t chunk = blockIdx.x; chunk < P.total_chunks; chunk += gridDim.x) {
    const int li = find_leaf(s_begin, P.n, chunk);
    const MagmaDotLeaf& L = P.leaf[li];
    const int64_t lo = (chunk - L.chunk_begin) * kChunk;
    const int64_t hi = (lo + kChunk < L.n ? lo + kChunk : L.n);
    float gm = 0.f, gg = 0.f, mm = 0.f;
    if (L.vec_ok) {
      for (int64_t i = lo + int64_t(threadIdx.x) * 8; i < hi; i += int64_t(blockDim.x) * 8) {
        float g[8], m[8];
        ld8(L.g, L.gdt, i, g);
        ld8(L.mu, L.mu_bf16 ? RF_BF16 : RF_F32, i, m);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float mt = __fadd_rn(__fmul_rn(P.s, g[k]), __fmul_rn(P.beta, m[k]));
          gm = fmaf(g[k], mt, gm);
          gg = fmaf(g[k], g[k], gg);
          mm = fmaf(mt, mt, mm);
        }
      }
    } else {
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float g = ld_as_float(L.g, L.gdt, i);
        const float m = ld_as_float(L.mu, L.mu_bf16 ? RF_BF16 : RF_F32, i);
        const float mt = __fadd_rn(__fmul_rn(P.s, g), __fmul_rn(P.beta, m));
        gm = fmaf(g, mt, gm);
        gg = fmaf(g, g, gg);
        mm = fmaf(mt, mt, mm);
      }
    }
    const float a = block_sum(gm, red);
    const float b = block_sum(gg, red);
    const float c = block_sum(mm, red);
    if (threadIdx.x == 0) {
      P.partials[3 * chunk] = a;
      P.partials[3 * chunk + 1] = b;
      P.partials[3 * chunk + 2] = c;
    }
  }
}

__global__ void __launch_bounds__(kEwThreads) k_magma_finalize(const __grid_constant__ MagmaFinLaunch P) {
  __shared__ float red[32];
  for (int li = blockIdx.x; li < P.n; li += gridDim.x) {
    const MagmaFinLeaf& L = P.leaf[li];
    float s3[3] = {0.f, 0.f, 0.f};
    for (int j = 0; j < 3; ++j) {
      float acc = 0.f;
      for (int64_t c = threadIdx.x; c < L.chunks; c += blockDim.x) acc += P.partials[3 * (L.chunk_begin + c) + j];
      s3[j] = block_sum(acc, red);
    }
    if (threadIdx.x == 0) {
      const float denom = fmaxf(__fmul_rn(__fsqrt_rn(s3[1]), __fsqrt_rn(s3[2])), 1e-12f);
      float cs = __fdiv_rn(s3[0], denom);
      if (cs != cs) cs = 0.f;  // nan_to_num(nan=0); +-inf are clipped below
      cs = fminf(fmaxf(cs, -1.f), 1.f);
      const float st = 1.f / (1.f + expf(-__fdiv_rn(cs, P.tau)));  // sigmoid(cos / tau)
      const float s_new = __fadd_rn(__fmul_rn(0.9f, *L.score), __fmul_rn(0.1f, st));
      *L.score = s_new;
      *L.factor = __fmul_rn(L.keep ? 1.f : 0.f, s_new);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// k_direction: mu <- s g + beta mu; out <- direction (custom orthogonalize_fn).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEwThreads) k_direction(const __grid_constant__ DirLaunch P) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].chunk_begin;
  __syncthreads();
  for (int64_t chunk = blockIdx.x; chunk < P.total_chunks; chunk += gridDim.x) {
    const int li = find_leaf(s_begin, P.n, chunk);
    const DirLeafDev& L = P.leaf[li];
    const int64_t lo = (chunk - L.chunk_begin) * kChunk;
    const int64_t hi = (lo + kChunk < L.n ? lo + kChunk : L.n);
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      const float g = ld_as_float(L.g, L.gdt, i);
      const float m = momentum_new(P.c, g, L.mu_bf16 ? ld_bf16(L.mu, i) : L.mu[i]);
      if (L.mu_bf16) sr_store1_bf16(L.mu, i, m, L.sr_seed);
      else L.mu[i] = m;
      L.out[i] = direction(P.c, g, m);
    }
  }
}

// ---------------------------------------------------------------------------
// k_tail: out = -lr * (shape_scale * O + decay * p) for gathered leaves.
// ---------------------------------------------------------------------------
// ds: the adaptive factor <d, O> (1 otherwise, which leaves o unchanged).
__device__ __forceinline__ float tail_one(const TailLeafDev& L, float neg_lr, float o, float p, float ds) {
  float u = __fmul_rn(__fmul_rn(ds, o), L.shape_scale);
  if (L.decay != 0.f) u = __fadd_rn(u, decay_term(L.decay_dt, L.decay, p));
  return __fmul_rn(neg_lr, u);
}

__global__ void __launch_bounds__(kEwThreads) k_tail(const __grid_constant__ TailLaunch P) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].chunk_begin;
  __syncthreads();
  for (int64_t chunk = blockIdx.x; chunk < P.total_chunks; chunk += gridDim.x) {
    const int li = find_leaf(s_begin, P.n, chunk);
    const TailLeafDev& L = P.leaf[li];
    const int64_t lo = (chunk - L.chunk_begin) * kChunk;
    const int64_t hi = (lo + kChunk < L.n ? lo + kChunk : L.n);
    const float ds = L.dev_scale ? *L.dev_scale : 1.f;
    if (L.vec_ok) {
      for (int64_t i = lo + int64_t(threadIdx.x) * 8; i < hi; i += int64_t(blockDim.x) * 8) {
        float o[8], p[8], u[8];
        ld8(L.o, L.odt, i, o);
        if (L.decay != 0.f) ld8(L.p, L.pdt, i, p);
#pragma unroll
        for (int k = 0; k < 8; ++k) u[k] = tail_one(L, P.neg_lr, o[k], L.decay != 0.f ? p[k] : 0.f, ds);
        st8(L.out, L.outdt, i, u);
      }
    } else {
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float p = L.decay != 0.f ? ld_as_float(L.p, L.pdt, i) : 0.f;
        st_from_float(L.out, L.outdt, i, tail_one(L, P.neg_lr, ld_as_float(L.o, L.odt, i), p, ds));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// adaptive (muon.py:272-282): per-chunk partial sums of d * O over each leaf
// (d with the reference's exact float32 direction formula), then one
// fixed-order sum per leaf.
// ---------------------------------------------------------------------------
template <int GDT>
__global__ void __launch_bounds__(kEwThreads) k_adaptive_dot(const __grid_constant__ AdaptiveLaunch P) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  __shared__ float red[32];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].chunk_begin;
  __syncthreads();
  for (int64_t chunk = blockIdx.x; chunk < P.total_chunks; chunk += gridDim.x) {
    const AdaptiveLeaf& L = P.leaf[find_leaf(s_begin, P.n, chunk)];
    if (L.gdt != GDT) continue;  // uniform per chunk: another launch covers it
    const int64_t lo = (chunk - L.chunk_begin) * kChunk;
    const int64_t hi = (lo + kChunk < L.n ? lo + kChunk : L.n);
    float s = 0.f;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      const float g = ld_as_float(L.g, GDT, i);
      float m;
      if (L.mu_bf16) {  // previous bf16 state: recompute, and store it here
        m = momentum_new(P.c, g, ld_bf16(L.mu, i));
        sr_store1_bf16(L.mu, i, m, L.sr_seed);
      } else {
        m = L.mu[i];
      }
      s += direction(P.c, g, m) * ld_as_float(L.o, L.odt, i);
    }
    s = block_sum(s, red);
    if (threadIdx.x == 0) P.partials[chunk] = s;
  }
}

__global__ void __launch_bounds__(kEwThreads) k_adaptive_finalize(const __grid_constant__ AdaptiveLaunch P,
                                                                  float* ip) {
  __shared__ float red[32];
  const AdaptiveLeaf& L = P.leaf[blockIdx.x];
  const int64_t nch = (L.n + kChunk - 1) / kChunk;
  float s = 0.f;
  for (int64_t k = threadIdx.x; k < nch; k += blockDim.x) s += P.partials[L.chunk_begin + k];
  s = block_sum(s, red);
  if (threadIdx.x == 0) ip[blockIdx.x] = s;
}

// ---------------------------------------------------------------------------
// apply_updates (utils.py:648-708) with the bf16 stochastic rounding of
// utils.py:342-371 (helpers at the top of this file).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEwThreads) k_apply(const __grid_constant__ ApplyLaunch P) {
  __shared__ int64_t s_begin[kMaxLeavesPerLaunch];
  for (int i = threadIdx.x; i < P.n; i += blockDim.x) s_begin[i] = P.leaf[i].chunk_begin;
  __syncthreads();
  for (int64_t chunk = blockIdx.x; chunk < P.total_chunks; chunk += gridDim.x) {
    const ApplyLeafDev& L = P.leaf[find_leaf(s_begin, P.n, chunk)];
    const int64_t lo = (chunk - L.chunk_begin) * kChunk;
    const int64_t hi = (lo + kChunk < L.n ? lo + kChunk : L.n);
    const bool sr = P.stochastic && L.pdt == RF_BF16;
    if (L.vec_ok) {
      for (int64_t i = lo + int64_t(threadIdx.x) * 8; i < hi; i += int64_t(blockDim.x) * 8) {
        float p[8], u[8];
        ld8(L.p, L.pdt, i, p);
        ld8(L.u, L.udt, i, u);
        uint64_t r0 = 0, r1 = 0;
        if (sr) {
          r0 = splitmix64_at(L.seed, uint64_t(i) >> 2);
          r1 = splitmix64_at(L.seed, (uint64_t(i) >> 2) + 1);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float sum = __fadd_rn(p[k], u[k]);
          // An SR result is exactly representable, so st8's conversion keeps it.
          p[k] = sr ? sr_bf16(sum, uint32_t(((k < 4 ? r0 : r1) >> (16 * (k & 3))) & 0xFFFFu)) : sum;
        }
        st8(L.out, L.pdt, i, p);
      }
    } else {
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float sum = __fadd_rn(ld_as_float(L.p, L.pdt, i), ld_as_float(L.u, L.udt, i));
        float v = sum;
        if (sr) {
          const uint64_t r = splitmix64_at(L.seed, uint64_t(i) >> 2);
          v = sr_bf16(sum, uint32_t((r >> (16 * (i & 3))) & 0xFFFFu));
        }
        st_from_float(L.out, L.pdt, i, v);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host launchers.
// ---------------------------------------------------------------------------
static int ew_grid(int64_t work, int ctas_per_sm = 8) {
  const int64_t cap = int64_t(num_sms()) * (ctas_per_sm > 0 ? ctas_per_sm : 8);
  return int(work < cap ? (work > 0 ? work : 1) : cap);
}

rf_status launch_magma_dot(const MagmaDotLaunch& P, cudaStream_t st) {
  if (P.total_chunks == 0) return RF_OK;
  k_magma_dot<<<ew_grid(P.total_chunks), kEwThreads, 0, st>>>(P);
  return check_launch("k_magma_dot");
}

rf_status launch_magma_finalize(const MagmaFinLaunch& P, cudaStream_t st) {
  if (P.n == 0) return RF_OK;
  k_magma_finalize<<<P.n, kEwThreads, 0, st>>>(P);
  return check_launch("k_magma_finalize");
}

rf_status launch_momentum_sumsq(const MomentumLaunch& P, int gdt, cudaStream_t st) {
  if (P.total_chunks == 0) return RF_OK;
  const int grid = ew_grid(P.total_chunks);
  if (gdt == RF_F32) k_momentum_sumsq<RF_F32><<<grid, kEwThreads, 0, st>>>(P);
  else if (gdt == RF_BF16) k_momentum_sumsq<RF_BF16><<<grid, kEwThreads, 0, st>>>(P);
  else k_momentum_sumsq<RF_F16><<<grid, kEwThreads, 0, st>>>(P);
  return check_launch("k_momentum_sumsq");
}

rf_status launch_norm_finalize(const MomentumLaunch& P, float* denom, float eps, cudaStream_t st) {
  if (P.total_mats == 0) return RF_OK;
  k_norm_finalize<<<ew_grid(P.total_mats), kEwThreads, 0, st>>>(P, denom, eps);
  return check_launch("k_norm_finalize");
}

template <int GDT>
static void launch_load_g(const LoadLaunch& P, int precision, int grid, cudaStream_t st) {
  if (precision == RF_NS_F16) k_ns_load<GDT, __half><<<grid, 256, 0, st>>>(P);
  else if (precision == RF_NS_BF16) k_ns_load<GDT, __nv_bfloat16><<<grid, 256, 0, st>>>(P);
  else k_ns_load<GDT, float><<<grid, 256, 0, st>>>(P);
}

rf_status launch_ns_load(const LoadLaunch& P, int gdt, int precision, cudaStream_t st) {
  const int64_t total = (P.mp / 64) * (P.np / 64) * P.group_mats;
  if (total == 0) return RF_OK;
  const int grid = int(total < int64_t(num_sms()) * 16 ? total : int64_t(num_sms()) * 16);
  if (gdt == RF_F32) launch_load_g<RF_F32>(P, precision, grid, st);
  else if (gdt == RF_BF16) launch_load_g<RF_BF16>(P, precision, grid, st);
  else launch_load_g<RF_F16>(P, precision, grid, st);
  return check_launch("k_ns_load");
}

rf_status launch_adamw(const AdamLaunch& P, cudaStream_t st) {
  if (P.total_chunks == 0) return RF_OK;
  k_adamw<<<ew_grid(P.total_chunks, P.max_ctas_per_sm), kEwThreads, 0, st>>>(P);
  return check_launch("k_adamw");
}

rf_status launch_direction(const DirLaunch& P, cudaStream_t st) {
  if (P.total_chunks == 0) return RF_OK;
  k_direction<<<ew_grid(P.total_chunks), kEwThreads, 0, st>>>(P);
  return check_launch("k_direction");
}

rf_status launch_adaptive_dot(const AdaptiveLaunch& P, int gdt, cudaStream_t st) {
  if (P.total_chunks == 0) return RF_OK;
  const int grid = ew_grid(P.total_chunks);
  if (gdt == RF_F32) k_adaptive_dot<RF_F32><<<grid, kEwThreads, 0, st>>>(P);
  else if (gdt == RF_BF16) k_adaptive_dot<RF_BF16><<<grid, kEwThreads, 0, st>>>(P);
  else k_adaptive_dot<RF_F16><<<grid, kEwThreads, 0, st>>>(P);
  return check_launch("k_adaptive_dot");
}

rf_status launch_adaptive_finalize(const AdaptiveLaunch& P, float* ip, cudaStream_t st) {
  if (P.n == 0) return RF_OK;
  k_adaptive_finalize<<<P.n, kEwThreads, 0, st>>>(P, ip);
  return check_launch("k_adaptive_finalize");
}

rf_status launch_apply(const ApplyLaunch& P, cudaStream_t st) {
  if (P.total_chunks == 0) return RF_OK;
  k_apply<<<ew_grid(P.total_chunks), kEwThreads, 0, st>>>(P);
  return check_launch("k_apply");
}

rf_status launch_tail(const TailLaunch& P, cudaStream_t st) {
  if (P.total_chunks == 0) return RF_OK;
  k_tail<<<ew_grid(P.total_chunks, P.max_ctas_per_sm), kEwThreads, 0, st>>>(P);
  return check_launch("k_tail");
}

}  // namespace rf

// Launch descriptors and launcher declarations shared by the kernels and the
// C-ABI layer.  Leaf tables are passed by value as kernel parameters.
#pragma once

#include "rf_common.cuh"

namespace rf {

constexpr int kEwThreads = 256;
constexpr int64_t kChunk = 8192;          // elements per CTA-chunk in multi-tensor kernels
constexpr int kMaxLeavesPerLaunch = 64;   // leaf-table entries per launch

int num_sms();

enum DirMode : int {
  kDirEmaNesterov = 0,
  kDirEma = 1,
  kDirHeavyBallNesterov = 2,
  kDirHeavyBall = 3,
  kDirIdentity = 4
};

struct MomentumCoeffs {
  float s;      // 1 - beta (ema) or 1 (heavy ball), utils.py:327-339
  float beta;
  float bc_mu;  // 1 - beta^(t+1) under Nesterov, else 1 - beta^t (ema only)
  float bc_g;   // 1 - beta^t (ema + Nesterov only)
  float rbc_mu, rbc_g;  // reciprocals, for the operand load (rounded to 16 bits afterwards)
  int mode;     // DirMode
};

struct MomentumLeaf {
  const void* g;
  float* mu;             // nullptr in kDirIdentity mode
  int64_t numel;         // elements per matrix (rows * cols)
  int64_t chunk_begin;   // first global chunk of this leaf
  int64_t mat_begin;     // first matrix index (within this launch) of this leaf
  int64_t scale_index;   // index of its first matrix in the per-matrix scale array
  int32_t chunks_per_mat;
  int32_t vec_ok;        // 16-byte aligned and numel % 8 == 0
  int32_t mu_bf16;       // mu stored as bfloat16: read it, leave the store to the operand load
};

struct MomentumLaunch {
  MomentumLeaf leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t total_chunks;
  int64_t total_mats;
  float* partials;         // [total_chunks] for this launch
  MomentumCoeffs c;
};

struct LoadLeaf {
  const void* g;
  const float* mu;
  int64_t rows, cols;        // leaf matrix (before the NS transpose)
  int64_t group_mat_begin;   // first matrix of this leaf within the group
  int64_t norm_index;        // index of its first matrix in the denominator array
  int32_t transposed;
  int32_t gdt;               // grad dtype; a launch handles the leaves of one dtype
  int32_t vec_ok;            // cols % 8 == 0 and 16-byte aligned grad / mu
  // bfloat16 momentum: mu holds the previous state; this load recomputes the
  // new momentum and, with store_mu, writes it back stochastically rounded.
  int32_t mu_bf16, store_mu;
  uint64_t sr_seed;
};

struct LoadLaunch {
  LoadLeaf leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t group_mats;  // matrices covered by this launch
  int64_t mp, np;      // padded NS dims
  const float* denom;  // per-matrix ||d||_F + eps
  float sx;            // power-of-two operand scale of this group
  void* x;             // X~0 for matrix 0 of this launch
  MomentumCoeffs c;
  // Optional [group_mats][mp] per-operand-row factors replacing 1 / denom
  // (AOL preconditioning); null: one denominator per matrix.
  const float* row_scale;
};

struct AdamCoeffs {
  float b1, b2, one_minus_b1, one_minus_b2, one_minus_b1_py;
  float bc1, bc1_next, bc2, eps, eps_root, neg_lr;
  int nesterov;
};
struct AdamLeafDev {
  const void* g;
  void* mu;
  void* nu;
  const void* p;
  void* out;
  int64_t n, chunk_begin;
  int32_t gdt, pdt, odt, decay_dt;
  int32_t vec_ok;  // 16-byte aligned buffers, n % 8 == 0 (and an 8-byte aligned mask)
  float decay;
  int32_t sdt;     // moment storage dtype: RF_F32, or RF_BF16 (stochastic rounding)
  uint64_t seed_mu, seed_nu;
  const uint8_t* mask;     // optional element-wise decay mask
  const float* scale_dev;  // optional device factor applied after the decay (Magma: keep * score)
  int32_t apply_mode;      // as in FinalLeaf: write p + u (the new parameter) instead of u
  uint64_t apply_seed;
};
struct AdamLaunch {
  AdamLeafDev leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t total_chunks;
  int max_ctas_per_sm;
  AdamCoeffs c;
};

struct DirLeafDev {
  const void* g;
  float* mu;  // bfloat16 storage when mu_bf16
  float* out;
  int64_t n, chunk_begin;
  int32_t gdt;
  int32_t mu_bf16;
  uint64_t sr_seed;
};
struct DirLaunch {
  DirLeafDev leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t total_chunks;
  MomentumCoeffs c;
};

struct TailLeafDev {
  const void* o;
  const void* p;
  void* out;
  int64_t n, chunk_begin;
  int32_t odt, pdt, outdt;
  int32_t vec_ok;  // 16-byte aligned buffers, n % 8 == 0
  float shape_scale, decay;
  const float* dev_scale;  // optional device factor applied to O first (adaptive)
  int32_t decay_dt;        // dtype decay * p is rounded to
};
struct TailLaunch {
  TailLeafDev leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t total_chunks;
  int max_ctas_per_sm;
  float neg_lr;
};

// --- Newton-Schulz GEMM stages ------------------------------------------------
// One call runs one of the three products of an NS iteration for every
// matrix of a shape group (padded to mp x np, multiples of 256):
//   kSyrkXXt : A~  = round(alpha * X~ X~^T)                    (upper tiles, mirrored)
//   kSyrkPoly: B~  = round(alpha * A~ A~ + beta * A~)          (upper tiles, mirrored)
//   kGemmBX  : X~' = round(alpha * B~ X~ + beta * X~)
//   kGemmBXFinal: O = (alpha * B~ X~ + beta * X~) * out_scale, written to each
//                 leaf in its own layout (transposed back when rows > cols),
//                 optionally with the fused tail -lr * (shape * O + decay * p).
enum NsStage : int { kSyrkXXt = 0, kSyrkPoly = 1, kGemmBX = 2, kGemmBXFinal = 3 };

struct FinalLeaf {
  void* out;
  const void* p;
  int64_t group_mat_begin;
  int32_t transposed;
  int32_t out_dtype, p_dtype;
  int32_t vec_ok;  // out / p 16-byte aligned and the leaf's row length % 8 == 0: vector epilogue
  float shape_scale, decay;
  int32_t decay_dt;  // dtype decay * p is rounded to (the parameter dtype, or RF_F32)
  const float* scale_dev;  // optional device factor applied after the decay (Magma: keep * score)
  // Fused parameter apply (utils.py:648-708): 0 off (out = the update);
  // 1: out = p + u rounded to the parameter dtype (nearest even); 2: the same
  // with bfloat16 stochastic rounding, noise of element i of apply_seed.
  int32_t apply_mode;
  uint64_t apply_seed;
};

struct NsGemmArgs {
  int stage;
  int precision;       // rf_ns_precision (operand storage)
  int reserve_sms;     // SMs the persistent grid leaves free
  int pdl;             // launch as a programmatic dependent of the previous stage on the stream
  int64_t G;           // matrices in the group
  int64_t m, n;        // true NS dims (m <= n)
  int64_t mp, np;      // padded dims
  const void* a_op;    // A operand [G][mp][K]  (X~ for XXt, A~ for Poly, B~ for BX)
  const void* b_op;    // B operand (X~ for XXt, A~ for Poly, X~ [G][mp][np] for BX)
  const void* aux;     // epilogue aux (A~ for Poly, X~ for BX)
  void* out;           // A~ / B~ / X~' (not used by the final stage)
  float alpha, beta;
  // final stage
  float out_scale;     // 1 / sx
  int fuse_tail;
  float neg_lr;
  int n_final;
  FinalLeaf final_leaf[kMaxLeavesPerLaunch];
};

rf_status launch_momentum_sumsq(const MomentumLaunch& P, int gdt, cudaStream_t st);
rf_status launch_norm_finalize(const MomentumLaunch& P, float* denom, float eps, cudaStream_t st);
rf_status launch_ns_load(const LoadLaunch& P, int gdt, int precision, cudaStream_t st);
rf_status launch_adamw(const AdamLaunch& P, cudaStream_t st);
rf_status launch_tail(const TailLaunch& P, cudaStream_t st);

// adaptive (muon.py:272-282): per leaf <d, O> over the whole leaf, d the
// Nesterov / bias-corrected direction recomputed from g and the updated mu.
struct AdaptiveLeaf {
  const void* g;
  float* mu;  // updated momentum; with mu_bf16 the previous bf16 state, stored here
  const void* o;
  int64_t n, chunk_begin;
  int32_t gdt, odt;
  int32_t mu_bf16;
  uint64_t sr_seed;
};
struct AdaptiveLaunch {
  AdaptiveLeaf leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t total_chunks;
  MomentumCoeffs c;
  float* partials;  // [total_chunks]
};
rf_status launch_adaptive_dot(const AdaptiveLaunch& P, int gdt, cudaStream_t st);

// apply_updates (utils.py:648-708).
struct ApplyLeafDev {
  const void* p;
  const void* u;
  void* out;
  int64_t n, chunk_begin;
  int32_t pdt, udt;
  int32_t vec_ok;  // 16-byte aligned buffers, n % 8 == 0
  uint64_t seed;
};
struct ApplyLaunch {
  ApplyLeafDev leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t total_chunks;
  int stochastic;
};
rf_status launch_apply(const ApplyLaunch& P, cudaStream_t st);

// Magma (src/rollfast/optim/magma.py:16-132): per leaf, partial sums over
// chunks of <g, mu_t>, |g|^2, |mu_t|^2 with mu_t = s g + beta mu_{t-1}
// recomputed from the previous state, then one fixed-order reduction per leaf
// giving the score EMA and the update factor keep * score.
struct MagmaDotLeaf {
  const void* g;
  const void* mu;      // previous first moment (float32, or bfloat16 storage)
  int64_t n, chunk_begin;
  int32_t gdt, mu_bf16, vec_ok;
};
struct MagmaDotLaunch {
  MagmaDotLeaf leaf[kMaxLeavesPerLaunch];
  int n;
  int64_t total_chunks;
  float s, beta;       // mu_t = s * g + beta * mu_{t-1}
  float* partials;     // [total_chunks][3]
};
struct MagmaFinLeaf {
  int64_t chunk_begin, chunks;
  float* score;        // the leaf's score, read and updated in place
  float* factor;       // out: keep * new score
  int32_t keep;
};
struct MagmaFinLaunch {
  MagmaFinLeaf leaf[kMaxLeavesPerLaunch];
  int n;
  float tau;
  const float* partials;
};
rf_status launch_magma_dot(const MagmaDotLaunch& P, cudaStream_t st);
rf_status launch_magma_finalize(const MagmaFinLaunch& P, cudaStream_t st);
rf_status launch_adaptive_finalize(const AdaptiveLaunch& P, float* ip, cudaStream_t st);

// Preconditioning variants (rf_precond.cu).  Reads A~ = sa X_F X_F^T of one
// sub-batch and either rewrites the per-matrix denominators (schatten,
// spectral) or returns per-row factors in `scratch` (aol, *row_scale).
// `basis` holds the Lanczos vectors (spectral): G * (min(64, m) + 1) * mp floats.
size_t precondition_scratch_bytes(int64_t G, int64_t mp);
rf_status launch_precondition(int mode, int precision, const void* A, int64_t G, int64_t m, int64_t mp, float sa,
                              const int64_t* begins, const int64_t* norm_index, int n_leaves, float* denom,
                              float eps, void* basis, size_t basis_bytes, void* scratch, size_t scratch_bytes,
                              const float** row_scale, cudaStream_t st);
rf_status launch_direction(const DirLaunch& P, cudaStream_t st);

// NS GEMM stage: tcgen05 path for 16-bit operands, SIMT path for fp32 (or
// when forced for cross-checking).
rf_status launch_ns_gemm(const NsGemmArgs& a, cudaStream_t st);
rf_status launch_ns_gemm_simt(const NsGemmArgs& a, cudaStream_t st);
rf_status launch_ns_gemm_tc(const NsGemmArgs& a, cudaStream_t st);

template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ float from_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_float<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Shared final-stage epilogue for one element (r, c) of matrix gm.
__device__ __forceinline__ int find_final_leaf(const NsGemmArgs& a, int64_t gm) {
  int lo = 0, hi = a.n_final - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (a.final_leaf[mid].group_mat_begin <= gm) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void final_store(const NsGemmArgs& a, const FinalLeaf& L, int64_t bi, int64_t r,
                                            int64_t c, float o) {
  // Leaf matrix is (m x n) when not transposed, (n x m) when transposed.
  const int64_t idx = bi * a.m * a.n + (L.transposed ? c * a.m + r : r * a.n + c);
  float v = o;
  if (a.fuse_tail) {
    const float pv = (L.decay != 0.f || L.apply_mode) ? ld_as_float(L.p, L.p_dtype, idx) : 0.f;
    v = __fmul_rn(o, L.shape_scale);
    if (L.decay != 0.f) v = __fadd_rn(v, decay_term(L.decay_dt, L.decay, pv));
    if (L.scale_dev) v = __fmul_rn(*L.scale_dev, v);
    v = __fmul_rn(a.neg_lr, v);
    if (L.apply_mode) {  // the new parameter: p + u in float32, then the parameter dtype
      st_rounded(L.out, L.out_dtype, idx, __fadd_rn(pv, v), L.apply_mode == 2, L.apply_seed);
      return;
    }
  }
  st_from_float(L.out, L.out_dtype, idx, v);
}

// Vector form of final_store for 32 consecutive leaf elements starting at
// linear index idx (a row run of a leaf, or a column run of a transposed
// leaf).  Requires FinalLeaf::vec_ok (16-byte aligned pointers, run start a
// multiple of 8).
__device__ __forceinline__ void final_store_run32(const NsGemmArgs& a, const FinalLeaf& L, int64_t idx,
                                                  const float* o) {
  float v[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = o[k];
  if (a.fuse_tail) {
    float pv[32];
    if (L.decay != 0.f || L.apply_mode) {
      if (L.p_dtype == RF_F32) {
        const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(L.p) + idx);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 x = q[j];
          pv[4 * j] = x.x; pv[4 * j + 1] = x.y; pv[4 * j + 2] = x.z; pv[4 * j + 3] = x.w;
        }
      } else {
        const uint4* q = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(L.p) + idx);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 u = q[j];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint16_t lo = uint16_t(w[h] & 0xFFFFu), hi = uint16_t(w[h] >> 16);
            if (L.p_dtype == RF_BF16) {
              pv[8 * j + 2 * h] = __bfloat162float(__ushort_as_bfloat16(lo));
              pv[8 * j + 2 * h + 1] = __bfloat162float(__ushort_as_bfloat16(hi));
            } else {
              pv[8 * j + 2 * h] = __half2float(__ushort_as_half(lo));
              pv[8 * j + 2 * h + 1] = __half2float(__ushort_as_half(hi));
            }
          }
        }
      }
    }
    const float fac = L.scale_dev ? *L.scale_dev : 1.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      float u = __fmul_rn(v[k], L.shape_scale);
      if (L.decay != 0.f) u = __fadd_rn(u, decay_term(L.decay_dt, L.decay, pv[k]));
      if (L.scale_dev) u = __fmul_rn(fac, u);
      v[k] = __fmul_rn(a.neg_lr, u);
    }
    if (L.apply_mode) {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = __fadd_rn(pv[k], v[k]);
      if (L.apply_mode == 2 && L.out_dtype == RF_BF16) {  // stochastic rounding, element idx + k's noise
        uint4* q = reinterpret_cast<uint4*>(static_cast<uint16_t*>(L.out) + idx);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t r0 = splitmix64_at(L.apply_seed, uint64_t(idx + 8 * j) >> 2);
          const uint64_t r1 = splitmix64_at(L.apply_seed, (uint64_t(idx + 8 * j) >> 2) + 1);
          uint32_t w[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint64_t r = h < 2 ? r0 : r1;
            const uint32_t lo = __float_as_uint(sr_bf16(v[8 * j + 2 * h], uint32_t((r >> (32 * (h & 1))) & 0xFFFFu)));
            const uint32_t hi =
                __float_as_uint(sr_bf16(v[8 * j + 2 * h + 1], uint32_t((r >> (32 * (h & 1) + 16)) & 0xFFFFu)));
            w[h] = (lo >> 16) | (hi & 0xFFFF0000u);
          }
          q[j] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        return;
      }
    }
  }
  if (L.out_dtype == RF_F32) {
    float4* q = reinterpret_cast<float4*>(static_cast<float*>(L.out) + idx);
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
    uint4* q = reinterpret_cast<uint4*>(static_cast<uint16_t*>(L.out) + idx);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float x0 = v[8 * j + 2 * h], x1 = v[8 * j + 2 * h + 1];
        uint16_t lo, hi;
        if (L.out_dtype == RF_BF16) {
          lo = __bfloat16_as_ushort(__float2bfloat16_rn(x0));
          hi = __bfloat16_as_ushort(__float2bfloat16_rn(x1));
        } else {
          lo = __half_as_ushort(__float2half_rn(x0));
          hi = __half_as_ushort(__float2half_rn(x1));
        }
        w[h] = uint32_t(lo) | (uint32_t(hi) << 16);
      }
      q[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Final-stage epilogue for one 32-column chunk held by a warp: lane l owns
// row row0 + l (columns col0..col0+31, values o[], already scaled to O).  A
// transposed leaf is stored along its rows, i.e. along the NS columns, so the
// warp's 32x32 block is transposed through `stg` (32 x 33 floats, per warp)
// and every lane writes one 32-element run.
__device__ __forceinline__ void final_chunk(const NsGemmArgs& a, const FinalLeaf& L, int64_t bi, int64_t row0,
                                           int64_t col0, int lane, const float* o, float* stg) {
  const int64_t mat = bi * a.m * a.n;
  if (!L.transposed) {
    const int64_t r = row0 + lane;
    if (r >= a.m) return;
    if (L.vec_ok && col0 + 32 <= a.n) {
      final_store_run32(a, L, mat + r * a.n + col0, o);
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (col0 + k < a.n) final_store(a, L, bi, r, col0 + k, o[k]);
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < 32; ++k) stg[lane * 33 + k] = o[k];
  __syncwarp();
  float t[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) t[i] = stg[i * 33 + lane];
  __syncwarp();
  const int64_t c = col0 + lane;
  if (c >= a.n) return;
  if (L.vec_ok && row0 + 32 <= a.m) {
    final_store_run32(a, L, mat + c * a.m + row0, t);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (row0 + i < a.m) final_store(a, L, bi, row0 + i, c, t[i]);
  }
}

}  // namespace rf

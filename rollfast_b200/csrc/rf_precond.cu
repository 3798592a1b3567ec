// Newton-Schulz preconditioning variants (orthogonalization.py:153-176,
// 233-250): "aol", "schatten" and "spectral", computed from the first
// iteration's A~ = sa * X_F X_F^T, where X_F = d / (||d||_F + eps) is the
// Frobenius-normalised operand the pipeline loads first.
//
// Each variant is a rescaling of the raw direction d followed by standard
// iterations:
//   aol       row i scaled by 1/sqrt(max(sum_j |A_ij|, 1e-8)), A = d d^T
//             (the rescaled first iteration of orthogonalization.py:153-163
//             equals the standard iteration on diag(s) d, since
//             diag(s) A diag(s) = (diag(s) d)(diag(s) d)^T);
//   schatten  d / sqrt(max(||d d^T||_F, 1e-8))  (166-176, same argument);
//   spectral  d / (||d||_2 + eps)  (247-250), ||d||_2^2 = lambda_max(d d^T).
// In terms of A_F = A~ / sa and den = ||d||_F + eps: d d^T = den^2 A_F.
// The clip 1e-8 of aol / schatten is the default of the reference's helper
// functions, which are called without an eps argument (189-201).
//
// lambda_max for "spectral" comes from Lanczos with full reorthogonalisation
// on A_F (min(64, m) steps; the top of a gradient's spectrum is clustered, so
// plain power iteration converges too slowly), then bisection on the
// tridiagonal matrix.  All kernels read A~ once per pass, row by row.
#include "rf_kernels.cuh"

namespace rf {
namespace pre {

constexpr int kMaxLanczos = 64;

struct PreArgs {
  int64_t begin[kMaxLeavesPerLaunch];       // first launch matrix of leaf i
  int64_t norm_index[kMaxLeavesPerLaunch];  // its first denominator slot
  int n;
  int mode;
  int64_t G, m, mp;
  const void* A;  // A~ [G][mp][mp]
  float inv_sa;
  float clip;     // 1e-8 (aol / schatten)
  float eps;      // user eps (spectral)
  float* denom;   // per-matrix denominators, updated in place
  float* rows;    // [G][mp]: aol row factors / schatten row sums of squares
  float* V;       // [G][K+1][mp] Lanczos basis
  float* W;       // [G][mp]
  float* T;       // [G][2 * (K+1)]: alpha[0..K), beta[0..K]
  int* keff;      // [G] Lanczos steps taken (breakdown stops early)
  int K;
};

__device__ __forceinline__ int64_t denom_slot(const PreArgs& a, int64_t gm) {
  int lo = 0, hi = a.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.begin[mid] <= gm) lo = mid;
    else hi = mid - 1;
  }
  return a.norm_index[lo] + (gm - a.begin[lo]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the block in a fixed order (deterministic); every thread gets it.
__device__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = lane < nw ? sh[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// 8 consecutive elements of a 16-bit or fp32 row as floats.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(h[k]);
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __bfloat1622float2(h[k]);
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}

// One warp per row of A~: aol row factors, or schatten row sums of squares.
template <typename T>
__global__ void __launch_bounds__(256) k_pre_rows(const __grid_constant__ PreArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t total = a.G * a.mp;
  for (int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5); row < total; row += int64_t(gridDim.x) * 8) {
    const int64_t g = row / a.mp, r = row - g * a.mp;
    float s = 0.f;
    if (r < a.m) {
      const T* p = static_cast<const T*>(a.A) + row * a.mp;
      for (int64_t j = int64_t(lane) * 8; j < a.mp; j += 256) {
        float v[8];
        load8<T>(p + j, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) s += a.mode == RF_PRECOND_AOL ? fabsf(v[k]) : v[k] * v[k];
      }
    }
    s = warp_sum(s);
    if (lane == 0) {
      if (a.mode == RF_PRECOND_AOL) {
        const float den = a.denom[denom_slot(a, g)];
        // 1 / sqrt(max(sum_j |A_ij|, clip)), with sum_j |A_ij| = den^2 * sum_j |A_F,ij|.
        a.rows[row] = r < a.m ? 1.f / sqrtf(fmaxf(s * a.inv_sa * den * den, a.clip)) : 0.f;
      } else {
        a.rows[row] = s;
      }
    }
  }
}

// Schatten: per matrix, ||A||_F = den^2 * sqrt(sum of row sums) / sa and the
// new denominator sqrt(max(||A||_F, clip)).
__global__ void __launch_bounds__(256) k_pre_schatten(const __grid_constant__ PreArgs a) {
  __shared__ float sh[32];
  const int64_t g = blockIdx.x;
  float s = 0.f;
  for (int64_t r = threadIdx.x; r < a.m; r += blockDim.x) s += a.rows[g * a.mp + r];
  s = block_sum(s, sh);
  if (threadIdx.x == 0) {
    const int64_t slot = denom_slot(a, g);
    const float den = a.denom[slot];
    const float fro = sqrtf(s) * a.inv_sa * den * den;
    a.denom[slot] = sqrtf(fmaxf(fro, a.clip));
  }
}

// Lanczos start: a fixed, positive, non-constant vector over the m real rows.
__global__ void __launch_bounds__(256) k_lz_init(const __grid_constant__ PreArgs a) {
  __shared__ float sh[32];
  const int64_t g = blockIdx.x;
  float* v = a.V + g * int64_t(a.K + 1) * a.mp;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) {
    const uint32_t h = uint32_t(i) * 2654435761u;
    const float x = i < a.m ? 0.5f + float(h >> 8) * (1.0f / 16777216.0f) : 0.f;
    v[i] = x;
    s += x * x;
  }
  s = block_sum(s, sh);
  const float inv = 1.f / sqrtf(s);
  for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) v[i] *= inv;
  if (threadIdx.x == 0) {
    a.keff[g] = a.K;
    a.T[g * 2 * (a.K + 1) + a.K] = 0.f;  // beta_0
  }
}

// w = A_F v_j, one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) k_lz_matvec(const __grid_constant__ PreArgs a, int j) {
  const int lane = threadIdx.x & 31;
  const int64_t total = a.G * a.mp;
  for (int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5); row < total; row += int64_t(gridDim.x) * 8) {
    const int64_t g = row / a.mp, r = row - g * a.mp;
    if (j >= a.keff[g]) continue;
    const float* v = a.V + (g * int64_t(a.K + 1) + j) * a.mp;
    float s = 0.f;
    if (r < a.m) {
      const T* p = static_cast<const T*>(a.A) + row * a.mp;
      for (int64_t c = int64_t(lane) * 8; c < a.mp; c += 256) {
        float x[8];
        load8<T>(p + c, x);
#pragma unroll
        for (int k = 0; k < 8; ++k) s += x[k] * v[c + k];
      }
    }
    s = warp_sum(s);
    if (lane == 0) a.W[row] = s * a.inv_sa;
  }
}

// One Lanczos step per matrix (one block): alpha_j, three-term recurrence,
// full reorthogonalisation against v_0..v_j, beta_{j+1}, v_{j+1}.
__global__ void __launch_bounds__(1024) k_lz_step(const __grid_constant__ PreArgs a, int j) {
  __shared__ float sh[32];
  const int64_t g = blockIdx.x;
  if (j >= a.keff[g]) return;
  float* V = a.V + g * int64_t(a.K + 1) * a.mp;
  float* w = a.W + g * a.mp;
  float* alpha = a.T + g * 2 * (a.K + 1);
  float* beta = alpha + a.K;  // beta[0..K]
  const float* vj = V + int64_t(j) * a.mp;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) s += vj[i] * w[i];
  const float al = block_sum(s, sh);
  const float bj = beta[j];
  const float* vp = j > 0 ? V + int64_t(j - 1) * a.mp : nullptr;
  for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) w[i] -= al * vj[i] + (vp ? bj * vp[i] : 0.f);
  __syncthreads();
  for (int q = 0; q <= j; ++q) {  // one Gram-Schmidt pass against the whole basis
    const float* vq = V + int64_t(q) * a.mp;
    float d = 0.f;
    for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) d += vq[i] * w[i];
    d = block_sum(d, sh);
    for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) w[i] -= d * vq[i];
    __syncthreads();
  }
  float n2 = 0.f;
  for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) n2 += w[i] * w[i];
  const float nb = sqrtf(block_sum(n2, sh));
  if (threadIdx.x == 0) alpha[j] = al;
  const bool stop = j + 1 >= a.K || !(nb > 1e-6f * (fabsf(al) + bj)) || nb == 0.f;
  if (stop) {
    if (threadIdx.x == 0) a.keff[g] = j + 1;
    return;
  }
  if (threadIdx.x == 0) beta[j + 1] = nb;
  const float inv = 1.f / nb;
  float* vn = V + int64_t(j + 1) * a.mp;
  for (int64_t i = threadIdx.x; i < a.mp; i += blockDim.x) vn[i] = w[i] * inv;
}

// Largest eigenvalue of each tridiagonal matrix by bisection on Sturm counts
// (double precision), then the spectral denominator den * sqrt(lambda) + eps.
__global__ void k_lz_finish(const __grid_constant__ PreArgs a) {
  const int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= a.G) return;
  const int n = a.keff[g];
  const float* alpha = a.T + g * 2 * (a.K + 1);
  const float* beta = alpha + a.K;
  double lo = 0.0, hi = 0.0;
  for (int i = 0; i < n; ++i) {
    const double r = (i > 0 ? fabs(double(beta[i])) : 0.0) + (i + 1 < n ? fabs(double(beta[i + 1])) : 0.0);
    lo = i == 0 ? alpha[i] - r : fmin(lo, alpha[i] - r);
    hi = i == 0 ? alpha[i] + r : fmax(hi, alpha[i] + r);
  }
  for (int it = 0; it < 200 && hi - lo > 1e-12 * fmax(1.0, fabs(hi)); ++it) {
    const double x = 0.5 * (lo + hi);
    int below = 0;  // eigenvalues < x
    double q = 1.0;
    for (int i = 0; i < n; ++i) {
      const double b2 = i > 0 ? double(beta[i]) * double(beta[i]) : 0.0;
      q = double(alpha[i]) - x - (i > 0 ? b2 / q : 0.0);
      if (q == 0.0) q = -1e-300;
      below += q < 0.0;
    }
    if (below >= n) hi = x;  // every eigenvalue lies below x
    else lo = x;
  }
  const int64_t slot = denom_slot(a, g);
  a.denom[slot] = a.denom[slot] * sqrtf(fmaxf(float(hi), 0.f)) + a.eps;
}

template <typename T>
rf_status launch_typed(PreArgs& a, cudaStream_t st) {
  const int64_t rows = a.G * a.mp;
  const unsigned row_blocks = unsigned(std::min<int64_t>(ceil_div(rows, 8), 148 * 32));
  if (a.mode == RF_PRECOND_AOL || a.mode == RF_PRECOND_SCHATTEN) {
    k_pre_rows<T><<<row_blocks, 256, 0, st>>>(a);
    RF_TRY(check_launch("k_pre_rows"));
    if (a.mode == RF_PRECOND_SCHATTEN) {
      k_pre_schatten<<<unsigned(a.G), 256, 0, st>>>(a);
      RF_TRY(check_launch("k_pre_schatten"));
    }
    return RF_OK;
  }
  k_lz_init<<<unsigned(a.G), 256, 0, st>>>(a);
  RF_TRY(check_launch("k_lz_init"));
  for (int j = 0; j < a.K; ++j) {
    k_lz_matvec<T><<<row_blocks, 256, 0, st>>>(a, j);
    RF_TRY(check_launch("k_lz_matvec"));
    k_lz_step<<<unsigned(a.G), 1024, 0, st>>>(a, j);
    RF_TRY(check_launch("k_lz_step"));
  }
  k_lz_finish<<<unsigned(ceil_div(a.G, 128)), 128, 0, st>>>(a);
  return check_launch("k_lz_finish");
}

}  // namespace pre

size_t precondition_scratch_bytes(int64_t G, int64_t mp) {
  return align_up(size_t(G) * mp * 4, 256) + align_up(size_t(G) * 2 * (pre::kMaxLanczos + 1) * 4, 256) +
         align_up(size_t(G) * 4, 256);
}

rf_status launch_precondition(int mode, int precision, const void* A, int64_t G, int64_t m, int64_t mp, float sa,
                              const int64_t* begins, const int64_t* norm_index, int n_leaves, float* denom,
                              float eps, void* basis, size_t basis_bytes, void* scratch, size_t scratch_bytes,
                              const float** row_scale, cudaStream_t st) {
  if (mode != RF_PRECOND_AOL && mode != RF_PRECOND_SCHATTEN && mode != RF_PRECOND_SPECTRAL)
    return fail(RF_EINVAL, "unknown preconditioning");
  if (n_leaves <= 0 || n_leaves > kMaxLeavesPerLaunch) return fail(RF_EINVAL, "preconditioning: bad leaf count");
  if (G > 0x7FFFFFFF) return fail(RF_EINVAL, "preconditioning: too many matrices");
  pre::PreArgs a{};
  for (int i = 0; i < n_leaves; ++i) {
    a.begin[i] = begins[i];
    a.norm_index[i] = norm_index[i];
  }
  a.n = n_leaves;
  a.mode = mode;
  a.G = G;
  a.m = m;
  a.mp = mp;
  a.A = A;
  a.inv_sa = 1.f / sa;
  a.clip = 1e-8f;
  a.eps = eps;
  a.denom = denom;
  a.K = int(std::min<int64_t>(pre::kMaxLanczos, m));
  uint8_t* s = static_cast<uint8_t*>(scratch);
  const size_t wbytes = align_up(size_t(G) * mp * 4, 256);
  const size_t tbytes = align_up(size_t(G) * 2 * (pre::kMaxLanczos + 1) * 4, 256);
  if (scratch_bytes < precondition_scratch_bytes(G, mp)) return fail(RF_EINVAL, "preconditioning: scratch too small");
  a.rows = reinterpret_cast<float*>(s);
  a.W = reinterpret_cast<float*>(s);
  a.T = reinterpret_cast<float*>(s + wbytes);
  a.keff = reinterpret_cast<int*>(s + wbytes + tbytes);
  if (mode == RF_PRECOND_SPECTRAL) {
    if (basis_bytes < size_t(G) * (a.K + 1) * mp * 4) return fail(RF_EINVAL, "preconditioning: basis too small");
    a.V = static_cast<float*>(basis);
  }
  *row_scale = mode == RF_PRECOND_AOL ? a.rows : nullptr;
  if (precision == RF_NS_F32) return pre::launch_typed<float>(a, st);
  if (precision == RF_NS_F16) return pre::launch_typed<__half>(a, st);
  return pre::launch_typed<__nv_bfloat16>(a, st);
}

}  // namespace rf

// CUDA-core (SIMT) Newton-Schulz GEMM stages.
//
// Used for the float32 precision mode (reference-grade parity with the
// reference's float32 NS, orthogonalization.py:227) and as an independent
// cross-check of the tcgen05 path on 16-bit operands.  Same stage semantics
// and epilogues as the tensor-core kernel (see NsGemmArgs).
#include "rf_kernels.cuh"

namespace rf {

namespace {

constexpr int SB = 64;   // tile edge
constexpr int SK = 16;   // k step
constexpr int ST = 256;  // threads, 4x4 outputs each

template <typename T>
__global__ void __launch_bounds__(ST) k_ns_simt(const __grid_constant__ NsGemmArgs a) {
  const int stage = a.stage;
  const bool sym = stage == kSyrkXXt || stage == kSyrkPoly;
  const int64_t I = blockIdx.y, J = blockIdx.x, gm = blockIdx.z;
  if (sym && J < I) return;
  const int64_t K = stage == kSyrkXXt ? a.np : a.mp;
  const int64_t ldc = sym ? a.mp : a.np;
  const T* A = static_cast<const T*>(a.a_op) + gm * a.mp * K;
  // sym: B has A's shape [mp][K]; BX: B is X~ [mp][np].
  const T* B = static_cast<const T*>(a.b_op) + gm * a.mp * (sym ? K : a.np);
  __shared__ float As[SK][SB + 4];
  __shared__ float Bs[SK][SB + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += SK) {
    for (int e = threadIdx.x; e < SB * SK; e += ST) {
      const int i = e / SK, kk = e % SK;
      As[kk][i] = to_float(A[(I * SB + i) * K + k0 + kk]);
      if (sym || stage == kSyrkXXt) {
        Bs[kk][i] = to_float(B[(J * SB + i) * K + k0 + kk]);
      }
    }
    if (!sym) {
      for (int e = threadIdx.x; e < SB * SK; e += ST) {
        const int kk = e / SB, j = e % SB;
        Bs[kk][j] = to_float(B[(k0 + kk) * a.np + J * SB + j]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) av[u] = As[kk][ty * 4 + u];
#pragma unroll
      for (int v = 0; v < 4; ++v) bv[v] = Bs[kk][tx * 4 + v];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
    }
    __syncthreads();
  }
  const T* aux = static_cast<const T*>(a.aux);
  T* out = static_cast<T*>(a.out);
  const int64_t mat_off = gm * a.mp * ldc;
  int fl = 0;
  if (stage == kGemmBXFinal) fl = find_final_leaf(a, gm);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int64_t r = I * SB + ty * 4 + u, c = J * SB + tx * 4 + v;
      float val = a.alpha * acc[u][v];
      if (sym) {
        if (c < r) continue;
        if (stage == kSyrkPoly) val = fmaf(a.beta, to_float(aux[mat_off + r * ldc + c]), val);
        const T tv = from_float<T>(val);
        out[mat_off + r * ldc + c] = tv;
        if (c != r) out[mat_off + c * ldc + r] = tv;
      } else {
        val = fmaf(a.beta, to_float(aux[mat_off + r * ldc + c]), val);
        if (stage == kGemmBX) {
          out[mat_off + r * ldc + c] = from_float<T>(val);
        } else if (r < a.m && c < a.n) {
          const FinalLeaf& L = a.final_leaf[fl];
          final_store(a, L, gm - L.group_mat_begin, r, c, val * a.out_scale);
        }
      }
    }
  }
}

}  // namespace

rf_status launch_ns_gemm_simt(const NsGemmArgs& a, cudaStream_t st) {
  const bool sym = a.stage == kSyrkXXt || a.stage == kSyrkPoly;
  dim3 grid(unsigned((sym ? a.mp : a.np) / SB), unsigned(a.mp / SB), unsigned(a.G));
  if (a.G > 65535) return fail(RF_EINVAL, "too many matrices in one NS group for the SIMT path");
  if (a.precision == RF_NS_F32) k_ns_simt<float><<<grid, ST, 0, st>>>(a);
  else if (a.precision == RF_NS_F16) k_ns_simt<__half><<<grid, ST, 0, st>>>(a);
  else k_ns_simt<__nv_bfloat16><<<grid, ST, 0, st>>>(a);
  return check_launch("k_ns_simt");
}

}  // namespace rf

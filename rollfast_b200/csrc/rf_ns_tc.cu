// Newton-Schulz GEMM stages on the 5th-generation tensor cores (sm_100a).
//
// One persistent, warp-specialised kernel serves the three products of a
// quintic NS iteration (orthogonalization.py:179-182) for every matrix of a
// shape group:
//   warp 0      TMA producer: 128x64 A tile + 256x64 B tile per stage into a
//               4-deep shared-memory ring (128-byte swizzle, no multicast)
//   warp 1      allocates 512 TMEM columns; lane 0 issues tcgen05.mma
//               (kind::f16, M=128 N=256 K=16, fp32 accumulate in TMEM) and
//               tcgen05.commit to release ring slots / publish accumulators
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from a
//               double-buffered accumulator (tile i+1's MMAs overlap tile i's
//               epilogue), fused polynomial / axpy / final-tail arithmetic
// The symmetric products X X^T and A A (A symmetric) visit only tiles that
// touch the upper triangle and store each element and its mirror once.
// Every mbarrier wait is bounded (globaltimer); a wait that gives up records
// an error code, drains its own in-flight copies/MMAs and frees TMEM.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <vector>

#include "rf_kernels.cuh"

namespace rf {

__device__ int g_tc_error = 0;  // first bounded-wait failure code (0 = none)

namespace tc {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;             // 16 KB
constexpr int B_BYTES = BN * BK * 2;             // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // 48 KB
constexpr int NUM_THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr int EPI_STAGE_BYTES = 4 * 32 * 33 * 4;  // per-warp 32x32 transpose buffers
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/ + EPI_STAGE_BYTES;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per wait

struct TcParams {
  NsGemmArgs a;
  int64_t total_tiles;
  int tiles_i;      // 128-row blocks per matrix
  int tiles_j;      // 256-col blocks per matrix
  int num_kb;       // 64-wide k blocks
  int sym;
  int b_mn_major;   // B operand is X~ [k][n] (n contiguous)
  uint32_t idesc;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}
// Bounded wait; returns false on timeout or when another role aborted.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) return false;
    }
  }
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// Programmatic dependent launch.  A stage launched with the programmatic
// stream serialization attribute may be scheduled while the previous stage
// drains; it touches global memory only after griddepcontrol.wait, which
// returns once the previous grid has completed and its writes are visible
// (at once for a launch without the attribute).  launch_dependents, issued by
// every CTA after that wait, lets the next stage's CTAs take the SMs this
// grid vacates and run their prologue (barrier init, TMEM allocation) there.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2),
// descriptor version 1, base offset 0 (tiles are 1024-byte aligned).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Tile index -> (matrix, row block I of 128, col block J of 256).
__device__ __forceinline__ void decode_tile(const TcParams& P, int64_t t, int64_t& g, int& I, int& J) {
  if (P.sym) {
    // Per matrix: row blocks I in [0, 2q), col blocks J in [I/2, q): q(q+1) tiles.
    const int q = P.tiles_j;
    const int64_t per = int64_t(q) * (q + 1);
    g = t / per;
    int rem = int(t - g * per);
    int i = 0;
    while (true) {
      const int cnt = q - (i >> 1);
      if (rem < cnt) break;
      rem -= cnt;
      ++i;
    }
    I = i;
    J = (i >> 1) + rem;
  } else {
    const int64_t per = int64_t(P.tiles_i) * P.tiles_j;
    g = t / per;
    const int rem = int(t - g * per);
    J = rem / P.tiles_i;  // column-of-tiles order: consecutive CTAs share the B column block
    I = rem - J * P.tiles_i;
  }
}

template <typename T>
struct Vec16;  // 8 x 16-bit <-> float
template <>
struct Vec16<__half> {
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 x = __half22float2(h[k]);
      f[2 * k] = x.x;
      f[2 * k + 1] = x.y;
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
    return u;
  }
};
template <>
struct Vec16<__nv_bfloat16> {
  static __device__ __forceinline__ void unpack(const uint4& u, float* f) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 x = __bfloat1622float2(h[k]);
      f[2 * k] = x.x;
      f[2 * k + 1] = x.y;
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
    return u;
  }
};

// 16-bit lane k (compile-time after unrolling) of 32 packed values.
__device__ __forceinline__ uint16_t lane16(const uint4 (&p)[4], int k) {
  const uint4& u = p[k >> 3];
  const int w = (k >> 1) & 3;
  const uint32_t word = w == 0 ? u.x : (w == 1 ? u.y : (w == 2 ? u.z : u.w));
  return (k & 1) ? uint16_t(word >> 16) : uint16_t(word & 0xFFFFu);
}

__device__ __forceinline__ void record_error(int code, volatile int* abort_flag) {
  *abort_flag = 1;
  atomicCAS(&g_tc_error, 0, code);
}

// The epilogue's second operand (A~ for the polynomial stage, X~ for the B X
// stages) for one 32-column chunk: 32 16-bit values of row row0 + lane.  The
// epilogue loads chunk c + 1 while it finishes chunk c, and a tile's first
// chunk before it waits for the accumulator, so these loads overlap the MMA
// and the previous chunk's stores instead of stalling each chunk.  Lanes
// whose symmetric chunk lies wholly below the diagonal load nothing.
template <typename T>
__device__ __forceinline__ void load_aux_chunk(const NsGemmArgs& a, bool sym, int64_t g, int64_t row0, int64_t col0,
                                               int lane, uint4 (&x)[4]) {
  const int64_t ldc = sym ? a.mp : a.np;
  const int64_t row = row0 + lane;
  if (sym && col0 + 31 < row) return;
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const T*>(a.aux) + g * a.mp * ldc + row * ldc + col0);
#pragma unroll
  for (int q = 0; q < 4; ++q) x[q] = p[q];
}

// 16-bit output blocks through the warp's shared staging buffer.  A lane
// holds one row of a 32x32 block (32 values in packed[]); stored directly,
// each store instruction would touch 32 rows.  Staged (17 words per row:
// conflict-free row writes and column gathers), the block leaves in 16-byte
// pieces that cover 8 rows per instruction, and its transpose (the mirrored
// block of a symmetric stage) in 4 such instructions instead of 32 2-byte
// stores.
__device__ __forceinline__ void stage_block16(uint32_t* s, int lane, const uint4 (&p)[4]) {
  __syncwarp();  // every lane has finished reading the previous block
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    s[lane * 17 + 4 * q + 0] = p[q].x;
    s[lane * 17 + 4 * q + 1] = p[q].y;
    s[lane * 17 + 4 * q + 2] = p[q].z;
    s[lane * 17 + 4 * q + 3] = p[q].w;
  }
  __syncwarp();
}
// Rows 0..31 of the staged block to out16[base + i * ldc + (0..31)].
__device__ __forceinline__ void store_block16(uint16_t* out16, int64_t base, int64_t ldc, const uint32_t* s,
                                              int lane) {
  const int q = lane & 3;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int i = t * 8 + (lane >> 2);
    const uint32_t* r = s + i * 17 + q * 4;
    *reinterpret_cast<uint4*>(out16 + base + int64_t(i) * ldc + q * 8) = make_uint4(r[0], r[1], r[2], r[3]);
  }
}
// Column j of the staged block to out16[base + j * ldc + (0..31)].
__device__ __forceinline__ void store_block16_t(uint16_t* out16, int64_t base, int64_t ldc, const uint32_t* s,
                                                int lane) {
  const int q = lane & 3;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int j = t * 8 + (lane >> 2);
    const int sh = (j & 1) * 16;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = (s[(q * 8 + 2 * e) * 17 + (j >> 1)] >> sh) & 0xFFFFu;
      const uint32_t hi = (s[(q * 8 + 2 * e + 1) * 17 + (j >> 1)] >> sh) & 0xFFFFu;
      w[e] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(out16 + base + int64_t(j) * ldc + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// One 32-column chunk of the epilogue.  The calling warp holds rows
// row0..row0+31 (lane = row - row0) of matrix g, columns col0..col0+31 of the
// accumulator in v[] and, for the stages with a second operand, that
// operand's chunk in xin[] (load_aux_chunk).  Stages: symmetric
// (upper-triangle store + mirror), general (fused a X + B X), final (O, or
// the fused tail, into the leaf).
template <typename T>
__device__ __forceinline__ void epilogue_chunk(const NsGemmArgs& a, bool sym, int64_t g, int64_t row0, int64_t col0,
                                               int lane, int fl, const float* v, const uint4 (&xin)[4], float* stg) {
  T* out = static_cast<T*>(a.out);
  const int64_t ldc = sym ? a.mp : a.np;
  const int64_t mat_off = g * a.mp * ldc;
  const int64_t row = row0 + lane;
  const int64_t rbase = mat_off + row * ldc + col0;
  float f[32];
  if (sym) {
    if (col0 + 31 < row) return;  // whole chunk below the diagonal (no warp-collective work follows)
    if (a.stage == kSyrkPoly) {
#pragma unroll
      for (int q = 0; q < 4; ++q) Vec16<T>::unpack(xin[q], f + 8 * q);
#pragma unroll
      for (int k = 0; k < 32; ++k) f[k] = fmaf(a.alpha, v[k], a.beta * f[k]);
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) f[k] = a.alpha * v[k];
    }
    // Round once; the direct and mirrored copies hold the same value.
    uint4 packed[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) packed[q] = Vec16<T>::pack(f + 8 * q);
    uint16_t* out16 = reinterpret_cast<uint16_t*>(out);
    if (col0 > row0) {
      // Above the diagonal (the same for every lane: row0 and col0 are
      // multiples of 32): the block and its mirror, staged.
      uint32_t* s32 = reinterpret_cast<uint32_t*>(stg);
      stage_block16(s32, lane, packed);
      store_block16(out16, mat_off + row0 * ldc + col0, ldc, s32, lane);
      store_block16_t(out16, mat_off + col0 * ldc + row0, ldc, s32, lane);
      return;
    }
    // The diagonal block: upper triangle and mirror element by element.
    if (col0 >= row) {
      uint4* op = reinterpret_cast<uint4*>(out + rbase);
#pragma unroll
      for (int q = 0; q < 4; ++q) op[q] = packed[q];
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (col0 + k >= row) out16[rbase + k] = lane16(packed, k);
    }
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int64_t c = col0 + k;
      if (c > row) out16[mat_off + c * ldc + row] = lane16(packed, k);
    }
    return;
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) Vec16<T>::unpack(xin[q], f + 8 * q);
#pragma unroll
  for (int k = 0; k < 32; ++k) f[k] = fmaf(a.alpha, v[k], a.beta * f[k]);
  if (a.stage == kGemmBX) {
    uint4 packed[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) packed[q] = Vec16<T>::pack(f + 8 * q);
    uint32_t* s32 = reinterpret_cast<uint32_t*>(stg);
    stage_block16(s32, lane, packed);
    store_block16(reinterpret_cast<uint16_t*>(out), mat_off + row0 * ldc + col0, ldc, s32, lane);
    return;
  }
  const FinalLeaf& L = a.final_leaf[fl];
#pragma unroll
  for (int k = 0; k < 32; ++k) f[k] *= a.out_scale;
  final_chunk(a, L, g - L.group_mat_begin, row0, col0, lane, f, stg);
}

template <typename T>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_ns_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ TcParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars[0..S) full, [S..2S) empty, [2S..2S+2) acc full, [2S+2..2S+4) acc empty
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* epi_stage = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256);  // 4 x 32x33 floats
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * STAGES), acce0 = smem_u32(bars + 2 * STAGES + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(accf0 + 8 * s, 1);
      mbar_init(acce0 + 8 * s, 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();
  allow_dependent_launch();
  const uint32_t tmem_base = *tmem_slot;
  const NsGemmArgs& a = P.a;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0;       // bit s: stage s has been filled at least once
      uint32_t last_par = 0;     // bit s: parity of the last fill of stage s
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < P.total_tiles; t += gridDim.x) {
        int64_t g;
        int I, J;
        decode_tile(P, t, g, I, J);
        for (int kb = 0; kb < P.num_kb; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag)) {
            record_error(kDevTimeoutProducer, abort_flag);
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8 * stage;
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          tma_load_3d(sa, &tmA, fb, kb * BK, I * BM, int(g));
          if (P.b_mn_major) {
#pragma unroll
            for (int q = 0; q < 4; ++q) tma_load_3d(sb + q * 8192, &tmB, fb, J * BN + q * 64, kb * BK, int(g));
          } else {
            tma_load_3d(sb, &tmB, fb, kb * BK, J * BN, int(g));
          }
          filled |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every copy this thread issued must land before the CTA exits.
      for (int s = 0; s < STAGES; ++s) {
        if (filled & (1u << s)) {
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(full0 + 8 * s, (last_par >> s) & 1u)) {
            if (globaltimer() - t0 > kTimeoutNs) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      int committed = -1;         // accumulator of the last tile commit
      uint32_t committed_par = 0;
      for (int64_t t = blockIdx.x; ok && t < P.total_tiles; t += gridDim.x) {
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1, abort_flag)) {
          record_error(kDevTimeoutMma, abort_flag);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < P.num_kb; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase, abort_flag)) {
            record_error(kDevTimeoutMma, abort_flag);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = sdesc(sa + k * 32, 16, 1024);
            const uint64_t bd = P.b_mn_major ? sdesc(sb + k * 2048, 8192, 1024) : sdesc(sb + k * 32, 16, 1024);
            mma_f16(d_tmem, ad, bd, P.idesc, (kb | k) != 0);
          }
          mma_commit(empty0 + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(accf0 + 8 * acc);
        committed = acc;
        committed_par = acc_phase;
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Drain: the last committed accumulator (hence all earlier MMAs) must
      // be complete before TMEM is released.
      if (committed >= 0) {
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(accf0 + 8 * committed, committed_par)) {
          if (globaltimer() - t0 > kTimeoutNs) break;
        }
      }
    }
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const bool has_aux = a.stage != kSyrkXXt;
    int acc = 0;
    uint32_t acc_phase = 0;
    float* stg = epi_stage + (warp - 2) * (32 * 33);
    for (int64_t t = blockIdx.x; t < P.total_tiles; t += gridDim.x) {
      int64_t g;
      int I, J;
      decode_tile(P, t, g, I, J);
      const int64_t row0 = int64_t(I) * BM + quarter * 32;
      const int64_t col_base = int64_t(J) * BN;
      uint4 xnext[4] = {};
      if (has_aux) load_aux_chunk<T>(a, P.sym, g, row0, col_base, lane, xnext);
      if (!mbar_wait(accf0 + 8 * acc, acc_phase, abort_flag)) {
        record_error(kDevTimeoutEpilogue, abort_flag);
        break;
      }
      tc_fence_after();
      int fl = 0;
      if (a.stage == kGemmBXFinal) fl = find_final_leaf(a, g);
      for (int ch = 0; ch < BN / 32; ++ch) {
        const uint4 xcur[4] = {xnext[0], xnext[1], xnext[2], xnext[3]};
        if (has_aux && ch + 1 < BN / 32) load_aux_chunk<T>(a, P.sym, g, row0, col_base + (ch + 1) * 32, lane, xnext);
        float v[32];
        __syncwarp();  // tcgen05.ld is warp-collective; lanes may have diverged on the diagonal
        tmem_ld32(tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + ch * 32), v);
        epilogue_chunk<T>(a, P.sym, g, row0, col_base + ch * 32, lane, fl, v, xcur, stg);
      }
      tc_fence_before();
      mbar_arrive(acce0 + 8 * acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ===========================================================================
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2): one 256x256 tile per
// pair.  CTA rank r loads A rows [128r, 128r+128) and its half of B
// (N columns [128r, 128r+128)) with ordinary (non-multicast) TMA loads that
// complete on the leader's full barrier; the leader's single MMA thread
// issues M=256 N=256 K=16 tcgen05.mma across both SMs' tensor cores, each
// SM accumulating its 128 rows in its own TMEM.  Commits are multicast to
// both CTAs' barriers; epilogue warps of both CTAs release the accumulator
// on the leader's barrier.  Per-SM operand traffic is half that of the
// single-CTA 128x256 tile for the same MMA rate.
// ===========================================================================
namespace tc2 {

#ifndef RF_TC2_STAGES
#define RF_TC2_STAGES 6
#endif
constexpr int BM = 128;                  // rows per CTA (256 per pair)
constexpr int BNH = 128;                 // B rows/cols per CTA (256 per pair)
constexpr int BK = 64, STAGES = RF_TC2_STAGES;  // pipeline depth (5, 6 and 7 measured alike)
constexpr int A_BYTES = BM * BK * 2;     // 16 KB
constexpr int B_BYTES = BNH * BK * 2;    // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256 + tc::EPI_STAGE_BYTES;
static_assert(SMEM_BYTES <= 232448, "dynamic shared memory per CTA is at most 227 KB");

using tc::kTimeoutNs;
using tc::smem_u32;
using tc::globaltimer;
using tc::mbar_init;
using tc::mbar_try_wait;
using tc::mbar_wait;
using tc::mbar_arrive_expect_tx;
using tc::tc_fence_before;
using tc::tc_fence_after;
using tc::sdesc;
using tc::tmem_ld32;
using tc::Vec16;
using tc::lane16;
using tc::record_error;
using tc::epilogue_chunk;

struct Tc2Params {
  NsGemmArgs a;
  int64_t total_tiles;  // 256x256 tiles (sym: upper triangle only)
  int tiles_i;          // 256-row blocks
  int tiles_j;          // 256-col blocks
  int num_kb;
  int sym;
  int b_mn_major;
  int group_rows;       // row blocks per tile group (decode_tile2)
  uint32_t idesc;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum));
}
// Arrive on the barrier at this shared offset in both CTAs of the pair once
// all prior tcgen05 operations of this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          bar)
      : "memory");
}

// Tile index -> (matrix, 256-row block I, 256-column block J), in an order
// that keeps the ~one wave of tiles in flight on a few operand panels, so
// that they share them in L2 as they advance through K together
// (G = P.group_rows):
//   general stages: groups of G row blocks, column by column within a group.
//     When B~ is too large to stay in L2 (8192-wide: 134 MB), G = 8: a wave
//     holds 8 B~ row panels and ~10 X~ column panels instead of every B~
//     panel.  When it fits, G = all row blocks: B~ stays in L2 across waves
//     and each X~ column panel is read once;
//   symmetric stages (upper triangle, J >= I), for the same large operands:
//     super-rows of G = 8 row blocks; within one, the columns from the
//     diagonal block outwards, each column's rows of the super-row up to the
//     diagonal (a wave touches 13 of the 32 panels of an 8192-row operand
//     instead of all of them).  Smaller ones (G = 0) go row by row, which
//     measured ~3% faster at 4096 rows.
// A matrix's tiles stay contiguous in t.
constexpr int kPanelGroup = 8;
constexpr int64_t kL2ResidentBytes = 48ll << 20;  // B~ at most this large stays in L2 across waves
__device__ __forceinline__ void decode_tile2(const Tc2Params& P, int64_t t, int64_t& g, int& I, int& J) {
  const int G = P.group_rows;
  if (P.sym) {
    const int q = P.tiles_j;  // square blocks
    const int64_t per = int64_t(q) * (q + 1) / 2;
    g = t / per;
    int rem = int(t - g * per);
    if (G == 0) {  // row by row: row block I holds q - I tiles
      int i = 0;
      while (rem >= q - i) {
        rem -= q - i;
        ++i;
      }
      I = i;
      J = i + rem;
      return;
    }
    int s0 = 0, gr = 0;
    while (true) {  // super-row holding rem: at most q / G + 1 steps
      gr = min(G, q - s0);
      const int cnt = gr * (gr + 1) / 2 + gr * (q - s0 - gr);
      if (rem < cnt) break;
      rem -= cnt;
      s0 += G;
    }
    const int tri = gr * (gr + 1) / 2;
    if (rem < tri) {  // columns s0 .. s0+gr-1: rows s0 .. J
      int jj = 0;
      while ((jj + 1) * (jj + 2) / 2 <= rem) ++jj;
      I = s0 + rem - jj * (jj + 1) / 2;
      J = s0 + jj;
    } else {  // columns right of the super-row's diagonal block: all gr rows
      rem -= tri;
      I = s0 + rem % gr;
      J = s0 + gr + rem / gr;
    }
  } else {
    const int64_t per = int64_t(P.tiles_i) * P.tiles_j;
    g = t / per;
    const int rem = int(t - g * per);
    const int grp = rem / (G * P.tiles_j);
    const int first = grp * G;
    const int gm = min(P.tiles_i - first, G);
    const int r2 = rem - grp * G * P.tiles_j;
    I = first + r2 % gm;
    J = r2 / gm;
  }
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    k_ns_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             const __grid_constant__ Tc2Params P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // [0,S) full (leader), [S,2S) empty, [2S,2S+2) acc full, [2S+2,2S+4) acc empty (leader)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* epi_stage = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256);  // 4 x 32x33 floats
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * STAGES), acce0 = smem_u32(bars + 2 * STAGES + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(accf0 + 8 * s, 1);
      mbar_init(acce0 + 8 * s, 8);  // 4 epilogue warps x 2 CTAs
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  grid_dependency_wait();
  allow_dependent_launch();
  const uint32_t tmem_base = *tmem_slot;
  const NsGemmArgs& a = P.a;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int64_t fills = 0;
      bool ok = true;
      for (int64_t t = pair; ok && t < P.total_tiles; t += npairs) {
        int64_t g;
        int I, J;
        decode_tile2(P, t, g, I, J);
        const int arow = I * 256 + int(rank) * BM;
        const int bcol = J * 256 + int(rank) * BNH;
        for (int kb = 0; kb < P.num_kb; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, abort_flag)) {
            record_error(kDevTimeoutProducer, abort_flag);
            ok = false;
            break;
          }
          const uint32_t fb_local = full0 + 8 * stage;
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * STAGE_BYTES);
          const uint32_t fb = map_to_rank(fb_local, 0);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          tma_load_3d_pair(sa, &tmA, fb, kb * BK, arow, int(g));
          if (P.b_mn_major) {
            tma_load_3d_pair(sb, &tmB, fb, bcol, kb * BK, int(g));
            tma_load_3d_pair(sb + 8192, &tmB, fb, bcol + 64, kb * BK, int(g));
          } else {
            tma_load_3d_pair(sb, &tmB, fb, kb * BK, bcol, int(g));
          }
          ++fills;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: wait until the MMA released each of the last (up to STAGES)
      // fills -- fill f is stage f % STAGES, and its release completes phase
      // f / STAGES of that stage's empty barrier -- so no copy into this
      // CTA's shared memory and no commit arrival on it is still pending.
      for (int64_t f = fills > STAGES ? fills - STAGES : 0; f < fills; ++f) {
        const uint32_t bar = empty0 + 8 * uint32_t(f % STAGES);
        const uint32_t par = uint32_t((f / STAGES) & 1);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(bar, par)) {
          if (globaltimer() - t0 > kTimeoutNs) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA) ----------------
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      int tiles_done = 0;
      for (int64_t t = pair; ok && t < P.total_tiles; t += npairs) {
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1, abort_flag)) {
          record_error(kDevTimeoutMma, abort_flag);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * 256);
        for (int kb = 0; kb < P.num_kb; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase, abort_flag)) {
            record_error(kDevTimeoutMma, abort_flag);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = sdesc(sa + k * 32, 16, 1024);
            const uint64_t bd = P.b_mn_major ? sdesc(sb + k * 2048, 8192, 1024) : sdesc(sb + k * 32, 16, 1024);
            mma_f16_pair(d_tmem, ad, bd, P.idesc, (kb | k) != 0);
          }
          mma_commit_pair(empty0 + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(accf0 + 8 * acc);
        ++tiles_done;
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Drain: wait until both CTAs' epilogues released the last (up to two)
      // tiles -- tile k used accumulator k % 2, and its release completes
      // phase k / 2 of that accumulator's empty barrier -- so every MMA and
      // every remote arrival has landed.
      for (int k = tiles_done > 2 ? tiles_done - 2 : 0; k < tiles_done; ++k) {
        const uint32_t bar = acce0 + 8 * uint32_t(k & 1);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(bar, uint32_t((k >> 1) & 1))) {
          if (globaltimer() - t0 > kTimeoutNs) break;
        }
      }
    }
  } else {
    // ---------------- Epilogue (warps 2..5 of both CTAs) ----------------
    const int quarter = warp & 3;
    const bool has_aux = a.stage != kSyrkXXt;
    int acc = 0;
    uint32_t acc_phase = 0;
    float* stg = epi_stage + (warp - 2) * (32 * 33);
    for (int64_t t = pair; t < P.total_tiles; t += npairs) {
      int64_t g;
      int I, J;
      decode_tile2(P, t, g, I, J);
      const int64_t row0 = int64_t(I) * 256 + int64_t(rank) * BM + quarter * 32;
      const int64_t col_base = int64_t(J) * 256;
      uint4 xnext[4] = {};
      if (has_aux) load_aux_chunk<T>(a, P.sym, g, row0, col_base, lane, xnext);
      if (!mbar_wait(accf0 + 8 * acc, acc_phase, abort_flag)) {
        record_error(kDevTimeoutEpilogue, abort_flag);
        break;
      }
      tc_fence_after();
      int fl = 0;
      if (a.stage == kGemmBXFinal) fl = find_final_leaf(a, g);
      for (int ch = 0; ch < 256 / 32; ++ch) {
        const uint4 xcur[4] = {xnext[0], xnext[1], xnext[2], xnext[3]};
        if (has_aux && ch + 1 < 256 / 32) load_aux_chunk<T>(a, P.sym, g, row0, col_base + (ch + 1) * 32, lane, xnext);
        float v[32];
        __syncwarp();
        tmem_ld32(tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * 256 + ch * 32), v);
        epilogue_chunk<T>(a, P.sym, g, row0, col_base + ch * 32, lane, fl, v, xcur, stg);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(acce0 + 8 * acc, 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still touch its TMEM / shared memory
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

}  // namespace tc2

// ---------------------------------------------------------------------------
// Host side: tensor maps (driver entry point fetched through the runtime, so
// the library does not link libcuda) and launch.
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D map over [G][rows][cols] 16-bit elements, box {64, box_rows, 1}.
rf_status make_map(CUtensorMap* map, const void* base, int precision, int64_t G, int64_t rows, int64_t cols,
                   uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(RF_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const CUtensorMapDataType dt =
      precision == RF_NS_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(G)};
  cuuint64_t strides[2] = {cuuint64_t(cols * 2), cuuint64_t(rows * cols * 2)};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RF_ECUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return RF_OK;
}

// One stage launch of NUM_THREADS-thread CTAs (the pair kernel's cluster
// shape is compiled in).  With pdl the launch carries the programmatic
// stream serialization attribute: the kernel may start while the previous
// kernel on the stream drains and orders itself with griddepcontrol.wait.
template <typename Kernel, typename Params>
rf_status launch_stage(Kernel kernel, unsigned grid, int smem, int pdl, cudaStream_t st, const CUtensorMap& mA,
                       const CUtensorMap& mB, const Params& P) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = size_t(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, mA, mB, P);
  if (e != cudaSuccess) return fail(RF_ECUDA, std::string("NS stage launch: ") + cudaGetErrorString(e));
  return RF_OK;
}

template <typename T>
rf_status launch_typed(const NsGemmArgs& a, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(k_ns_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return fail(RF_ECUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(attr_err));

  TcParams P;
  P.a = a;
  const bool sym = a.stage == kSyrkXXt || a.stage == kSyrkPoly;
  P.sym = sym;
  P.b_mn_major = sym ? 0 : 1;
  P.tiles_i = int(a.mp / BM);
  P.tiles_j = int((sym ? a.mp : a.np) / BN);
  const int64_t K = a.stage == kSyrkXXt ? a.np : a.mp;
  P.num_kb = int(K / BK);
  P.total_tiles = sym ? a.G * int64_t(P.tiles_j) * (P.tiles_j + 1) : a.G * int64_t(P.tiles_i) * P.tiles_j;
  const uint32_t fmt = a.precision == RF_NS_F16 ? 0u : 1u;
  P.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(P.b_mn_major) << 16) | (uint32_t(BN >> 3) << 17) |
            (uint32_t(BM >> 4) << 24);

  CUtensorMap mA, mB;
  // A operand: [G][mp][K] rows of 128; B operand: K-major [G][mp][K] rows of
  // 256, or X~ [G][mp][np] read as 64(k) x 64(n) boxes.
  RF_TRY(make_map(&mA, a.a_op, a.precision, a.G, a.mp, K, BM));
  if (sym) RF_TRY(make_map(&mB, a.b_op, a.precision, a.G, a.mp, K, BN));
  else RF_TRY(make_map(&mB, a.b_op, a.precision, a.G, a.mp, a.np, 64));

  int64_t cap = num_sms() - a.reserve_sms;
  if (cap < 1) cap = 1;
  const int64_t grid = P.total_tiles < cap ? P.total_tiles : cap;
  RF_TRY(launch_stage(k_ns_tc<T>, unsigned(grid), SMEM_BYTES, a.pdl, st, mA, mB, P));
  return check_launch("k_ns_tc");
}

}  // namespace tc

namespace tc {
namespace tc2 {
template <typename T>
rf_status launch_typed(const NsGemmArgs& a, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(k_ns_tc2<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return fail(RF_ECUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(attr_err));
  Tc2Params P;
  P.a = a;
  const bool sym = a.stage == kSyrkXXt || a.stage == kSyrkPoly;
  P.sym = sym;
  P.b_mn_major = sym ? 0 : 1;
  P.tiles_i = int(a.mp / 256);
  P.tiles_j = int((sym ? a.mp : a.np) / 256);
  const int64_t K = a.stage == kSyrkXXt ? a.np : a.mp;
  P.num_kb = int(K / BK);
  P.total_tiles = sym ? a.G * int64_t(P.tiles_j) * (P.tiles_j + 1) / 2 : a.G * int64_t(P.tiles_i) * P.tiles_j;
  const bool large = a.mp * a.mp * 2 > kL2ResidentBytes;
  P.group_rows = large ? kPanelGroup : (sym ? 0 : P.tiles_i);
  const uint32_t fmt = a.precision == RF_NS_F16 ? 0u : 1u;
  P.idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(P.b_mn_major) << 16) | (uint32_t(256 >> 3) << 17) |
            (uint32_t(256 >> 4) << 24);
  CUtensorMap mA, mB;
  RF_TRY(tc::make_map(&mA, a.a_op, a.precision, a.G, a.mp, K, BM));
  if (sym) RF_TRY(tc::make_map(&mB, a.b_op, a.precision, a.G, a.mp, K, BNH));
  else RF_TRY(tc::make_map(&mB, a.b_op, a.precision, a.G, a.mp, a.np, 64));
  static int64_t pairs_max = [] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(num_sms()), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, k_ns_tc2<T>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    return int64_t(n);
  }();
  int64_t cap = pairs_max - (a.reserve_sms + 1) / 2;
  if (cap < 1) cap = 1;
  const int64_t pairs = P.total_tiles < cap ? P.total_tiles : cap;
  RF_TRY(launch_stage(k_ns_tc2<T>, unsigned(2 * pairs), SMEM_BYTES, a.pdl, st, mA, mB, P));
  return check_launch("k_ns_tc2");
}
}  // namespace tc2
}  // namespace tc

// Tensor-core kernel choice: the CTA-pair kernel when it has a full wave of
// 256x256 tiles, otherwise the single-CTA kernel (twice as many 128x256
// tiles for small groups).  ROLLFAST_NS_KERNEL=1|2 forces one.
static int tc_variant(const NsGemmArgs& a) {
  const char* e = getenv("ROLLFAST_NS_KERNEL");
  const int forced = e ? atoi(e) : 0;
  if (forced == 1 || forced == 2) return forced;
  const bool sym = a.stage == kSyrkXXt || a.stage == kSyrkPoly;
  const int64_t q = a.mp / 256;
  const int64_t tiles2 = sym ? a.G * q * (q + 1) / 2 : a.G * q * (a.np / 256);
  return tiles2 >= num_sms() / 2 ? 2 : 1;
}

rf_status launch_ns_gemm_tc(const NsGemmArgs& a, cudaStream_t st) {
  if (a.mp % 256 || a.np % 256) return fail(RF_EINVAL, "tcgen05 NS path needs dims padded to 256");
  if (a.G > 0x7FFFFFFF) return fail(RF_EINVAL, "group too large");
  const int v = tc_variant(a);
  if (a.precision == RF_NS_F16) return v == 2 ? tc::tc2::launch_typed<__half>(a, st) : tc::launch_typed<__half>(a, st);
  if (a.precision == RF_NS_BF16)
    return v == 2 ? tc::tc2::launch_typed<__nv_bfloat16>(a, st) : tc::launch_typed<__nv_bfloat16>(a, st);
  return fail(RF_EINVAL, "tcgen05 path takes 16-bit operands");
}

// ---------------------------------------------------------------------------
// Launch profiling (rf_profile_begin / rf_profile_end).
// ---------------------------------------------------------------------------
namespace {
struct ProfRec {
  cudaEvent_t start, stop;
  double alg, exec;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRec> g_prof;

void stage_flops(const NsGemmArgs& a, double& alg, double& exec) {
  const double G = double(a.G), m = double(a.m), n = double(a.n), mp = double(a.mp), np = double(a.np);
  if (a.stage == kSyrkXXt || a.stage == kSyrkPoly) {
    const double k = a.stage == kSyrkXXt ? n : m;
    const double kp = a.stage == kSyrkXXt ? np : mp;
    alg = 2.0 * G * m * m * k;
    if (a.precision == RF_NS_F32) {
      const double q = mp / 64.0;
      exec = 2.0 * G * (q * (q + 1) / 2.0) * 64.0 * 64.0 * kp;
    } else {
      const double q = mp / 256.0;
      exec = 2.0 * G * (q * (q + 1)) * 128.0 * 256.0 * kp;
    }
  } else {
    alg = 2.0 * G * m * m * n;
    exec = 2.0 * G * mp * mp * np;
  }
}
}  // namespace

rf_status launch_ns_gemm(const NsGemmArgs& a, cudaStream_t st) {
  ProfRec rec{};
  bool prof = false;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    prof = g_prof_on;
  }
  if (prof) {
    if (cudaEventCreate(&rec.start) != cudaSuccess || cudaEventCreate(&rec.stop) != cudaSuccess)
      return fail(RF_ECUDA, "cudaEventCreate failed");
    cudaEventRecord(rec.start, st);
  }
  rf_status r = a.precision == RF_NS_F32 ? launch_ns_gemm_simt(a, st) : launch_ns_gemm_tc(a, st);
  if (prof) {
    cudaEventRecord(rec.stop, st);
    stage_flops(a, rec.alg, rec.exec);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof.push_back(rec);
  }
  return r;
}

}  // namespace rf

extern "C" rf_status rf_profile_begin(void) {
  std::lock_guard<std::mutex> lk(rf::g_prof_mu);
  for (auto& r : rf::g_prof) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  rf::g_prof.clear();
  rf::g_prof_on = true;
  return RF_OK;
}

extern "C" rf_status rf_profile_end(double* gemm_ms, int64_t* launches, double* alg, double* exec) {
  if (!gemm_ms || !launches || !alg || !exec) return rf::fail(RF_EINVAL, "null output pointer");
  std::lock_guard<std::mutex> lk(rf::g_prof_mu);
  rf::g_prof_on = false;
  double ms = 0, a = 0, e = 0;
  for (auto& r : rf::g_prof) {
    cudaError_t ce = cudaEventSynchronize(r.stop);
    if (ce != cudaSuccess) return rf::fail(RF_ECUDA, std::string("profile sync: ") + cudaGetErrorString(ce));
    float t = 0.f;
    cudaEventElapsedTime(&t, r.start, r.stop);
    ms += t;
    a += r.alg;
    e += r.exec;
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  *gemm_ms = ms;
  *launches = int64_t(rf::g_prof.size());
  *alg = a;
  *exec = e;
  rf::g_prof.clear();
  return RF_OK;
}

namespace rf {

// Reads and clears the device error word (synchronises the device).
rf_status take_device_error() {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
  if (e != cudaSuccess) return fail(RF_ECUDA, std::string("reading device error word: ") + cudaGetErrorString(e));
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
    return fail(RF_ETIMEOUT, "a bounded device-side wait gave up (code " + std::to_string(v) + ")");
  }
  return RF_OK;
}

// Stream-ordered copy of the tensor-core kernels' error word to *dst.
rf_status snapshot_device_error(int32_t* dst, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(dst, g_tc_error, sizeof(int), 0, cudaMemcpyDefault, st);
  if (e != cudaSuccess) return fail(RF_ECUDA, std::string("copying device error word: ") + cudaGetErrorString(e));
  return RF_OK;
}

}  // namespace rf

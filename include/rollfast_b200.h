/*
 * rollfast_b200 -- C ABI of the B200-native Muon update hot path.
 *
 * Every entry point is stream-ordered and asynchronous, takes plain device
 * pointers and sizes, never allocates device memory and never aborts: it
 * returns an rf_status and keeps a thread-local message for rf_last_error().
 * The caller owns every buffer (inputs, outputs and the workspace sized by
 * the *_workspace_size queries).
 *
 * The entry points replace the per-leaf work of the reference's Optax
 * transforms (RhizomeResearch/rollfast, paths relative to its root):
 *   rf_muon_update          <- scale_by_muon.update_fn + scale_by_shape +
 *                              add_decayed_weights + scale_by_learning_rate
 *                              for the Muon branch (src/rollfast/optim/muon.py:225-330,
 *                              130-137, 390-393, 462-467)
 *   rf_newton_schulz        <- orthogonalize_via_newton_schulz / quintic_newton_schulz,
 *                              the `orthogonalize_fn` plugin seam
 *                              (src/rollfast/optim/orthogonalization.py:211-305)
 *   rf_adamw_update         <- scale_by_adam.update_fn + add_decayed_weights +
 *                              scale_by_learning_rate (src/rollfast/optim/adam.py:123-233, 380-404)
 *   rf_muon_tail            <- scale_by_shape + add_decayed_weights + scale_by_learning_rate
 *                              applied to gathered orthogonalised leaves (muon.py:130-137, 390-393, 466)
 *   rf_apply_updates        <- apply_updates with bf16 stochastic rounding (src/rollfast/utils.py:342-371, 648-708)
 * Without a reference counterpart: rf_newton_schulz_noalloc (static
 * workspace), and the peer transport of the multi-GPU sharded update
 * (rf_ipc_*, rf_peer_copy, rf_flags_*; rf_ipc_open maps, but does not
 * allocate, another process's memory).
 * A JAX integration registers these as XLA FFI custom calls; a ctypes
 * binding (rollfast_b200/_lib.py) is the host used in this repository.
 */
#ifndef ROLLFAST_B200_H_
#define ROLLFAST_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum rf_status {
  RF_OK = 0,
  RF_EINVAL = 1,    /* bad shape / dtype / null pointer / too-small workspace */
  RF_ECUDA = 2,     /* CUDA launch or driver error (message in rf_last_error) */
  RF_ETIMEOUT = 3,  /* a bounded device-side wait gave up; results invalid */
  RF_ENOTSUP = 4    /* option outside the supported hot path */
} rf_status;

typedef enum rf_dtype { RF_F32 = 0, RF_BF16 = 1, RF_F16 = 2 } rf_dtype;

typedef enum rf_accumulator { RF_EMA = 0, RF_HEAVY_BALL = 1 } rf_accumulator;

/* Newton-Schulz operand precision: 16-bit tensor-core operands (fp32
 * accumulate in TMEM) or a float32 path for reference-grade parity. */
typedef enum rf_ns_precision { RF_NS_F16 = 0, RF_NS_BF16 = 1, RF_NS_F32 = 2 } rf_ns_precision;

/* One Muon leaf, already in the reference's (batch, reduction, output)
 * layout (dimension_numbers.py:312-359): a contiguous [batch][rows][cols]
 * array.  Newton-Schulz runs on the rows x cols matrices, transposed when
 * rows > cols (orthogonalization.py:228-231). */
typedef struct rf_muon_leaf {
  const void* grad;   /* [batch][rows][cols], grad_dtype */
  float* mu;          /* [batch][rows][cols] momentum (mu_dtype storage), updated in place */
  const void* param;  /* [batch][rows][cols], param_dtype; may be NULL when decay == 0 */
  void* out;          /* [batch][rows][cols], out_dtype: the update (or O when the tail is deferred) */
  int64_t batch, rows, cols;
  int32_t grad_dtype, param_dtype, out_dtype;
  float shape_scale;  /* muon.py:79-100 factor for this leaf */
  float decay;        /* weight decay for this leaf (0 when masked out) */
  int32_t skip_ns;    /* 1: this rank does not own the leaf (multi-GPU); momentum/NS skipped */
  /* RF_F32, or RF_BF16: momentum stored as bfloat16 (mu_dtype, muon.py:207-210).
   * The step then reads the bf16 state, forms the new momentum and the
   * direction in float32, and stores the new momentum stochastically rounded
   * (utils.py:342-371, 412-425) with SplitMix64 noise from sr_seed; the
   * reference draws JAX Threefry bits, so the stored state agrees with it in
   * distribution, not bit for bit. */
  int32_t mu_dtype;
  uint64_t sr_seed;
  /* 0: decay * p is rounded to the parameter dtype (optax add_decayed_weights
   * with a Python-float weight decay, weakly typed); 1: formed in float32 (a
   * schedule whose value is a float32 array, strongly typed). */
  int32_t decay_in_f32;
  /* Magma (src/rollfast/optim/magma.py:16-132), NULL when off: the leaf's
   * score (one float32 in device memory, read and updated in place: score <-
   * 0.9 score + 0.1 sigmoid(cos(g, mu_t) / magma_tau)), and its Bernoulli
   * draw for this step (magma_keep 0 or 1); the leaf's update is scaled by
   * magma_keep * score after the decay and before the learning rate. */
  float* magma_score;
  int32_t magma_keep;
  /* Fused parameter apply (utils.py:648-708; needs fuse_tail and param):
   * 0: `out` receives the update; 1: `out` (param_dtype, may alias param)
   * receives the new parameter p + u, rounded to nearest even; 2: the same
   * with bfloat16 stochastic rounding (noise of element i of apply_seed's
   * SplitMix64 stream, as rf_apply_updates draws it for a leaf with that
   * seed).  Saves writing the float32 update and reading it back. */
  int32_t apply_mode;
  uint64_t apply_seed;
} rf_muon_leaf;

/* Newton-Schulz preconditioning (orthogonalization.py:24, 153-176, 233-250). */
typedef enum rf_preconditioning {
  RF_PRECOND_FROBENIUS = 0, /* X / (||X||_F + eps) */
  RF_PRECOND_SPECTRAL = 1,  /* X / (||X||_2 + eps) */
  RF_PRECOND_AOL = 2,       /* first iteration on diag(s) X, s_i = 1/sqrt(max(sum_j |(X X^T)_ij|, 1e-8)) */
  RF_PRECOND_SCHATTEN = 3   /* first iteration on X / sqrt(max(||X X^T||_F, 1e-8)) */
} rf_preconditioning;

typedef struct rf_muon_params {
  float beta;            /* muon.py:402 */
  float eps;             /* muon.py:403, Frobenius normaliser epsilon */
  int32_t count;         /* state.count before this step (0-based) */
  int32_t nesterov;      /* muon.py:408 */
  int32_t accumulator;   /* rf_accumulator */
  int32_t ns_steps;      /* iterations when coeffs is a single (a,b,c) triple */
  /* 0: coeffs is one (a,b,c) triple applied ns_steps times (fori_loop,
   * orthogonalization.py:253-260); n > 0: coeffs is an ordered (n,3)
   * schedule and exactly n iterations run (lax.scan, orthogonalization.py:262-269). */
  int32_t n_coeff_rows;
  const float* coeffs;   /* HOST pointer: max(1, n_coeff_rows) * 3 floats (a,b,c) */
  int32_t precision;     /* rf_ns_precision */
  float lr;              /* learning rate at this step (scale_by_learning_rate) */
  int32_t fuse_tail;     /* 1: out = -lr*(scale*O + decay*p); 0: out = O (leaf layout) */
  /* Optional second stream (NULL: everything on `stream`).  The HBM-bound
   * preparation of the next shape sub-batch (momentum, norms, operand load)
   * then runs on it while the current sub-batch's Newton-Schulz GEMMs run on
   * `stream`; ordering is kept with events and all work is ordered before
   * later work on `stream` when the call returns.  Needs a workspace sized
   * with pipelined = 1. */
  void* aux_stream;
  /* SMs the GEMM kernels leave free for concurrent kernels (e.g. a
   * collective or the tail on another stream); 0 = use every SM. */
  int32_t reserve_sms;
  int32_t preconditioning;  /* rf_preconditioning (muon.py:410) */
  /* 1: O <- <d, O> O per leaf before the tail (muon.py:272-282), d the
   * Nesterov / bias-corrected direction; the NS final epilogue then writes O
   * and a separate pass applies the factor and the tail. */
  int32_t adaptive;
  float magma_tau;  /* Magma temperature (muon.py:178), used by leaves with a magma_score */
} rf_muon_params;

/* Bytes of workspace rf_muon_update needs for these leaves and precision
 * (pipelined != 0: two sub-batch regions, for use with an aux stream). */
rf_status rf_muon_workspace_size(const rf_muon_leaf* leaves, int32_t n_leaves, int32_t precision,
                                 int32_t pipelined, size_t* bytes);

/* Full Muon-branch step for n_leaves leaves: momentum (EMA / heavy-ball,
 * Nesterov, bias correction), Frobenius normalisation, quintic Newton-Schulz,
 * and (fuse_tail) shape scale + decoupled decay + learning-rate scale.
 * Leaves of equal matrix shape are batched into one grouped launch per GEMM. */
rf_status rf_muon_update(const rf_muon_leaf* leaves, int32_t n_leaves, const rf_muon_params* params,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Momentum step alone, for a caller-supplied orthogonalize_fn: updates mu in
 * place and writes the Nesterov / bias-corrected direction (fp32, leaf
 * layout) to each leaf's `out` (utils.py:565-645; muon.py:240-256). */
rf_status rf_muon_direction(const rf_muon_leaf* leaves, int32_t n_leaves, const rf_muon_params* params,
                            void* stream);

/* The orthogonalize_fn seam: out = NS(x) over [batch][rows][cols]
 * (coeffs / n_coeff_rows / ns_steps as in rf_muon_params). */
rf_status rf_newton_schulz_workspace_size(int64_t batch, int64_t rows, int64_t cols,
                                          int32_t precision, size_t* bytes);
rf_status rf_newton_schulz(const void* x, int32_t x_dtype, void* out, int32_t out_dtype,
                           int64_t batch, int64_t rows, int64_t cols, const float* coeffs,
                           int32_t n_coeff_rows, int32_t ns_steps, float eps, int32_t preconditioning,
                           int32_t precision, void* workspace, size_t workspace_bytes, void* stream);

/* rf_newton_schulz for callers that cannot allocate device memory (no
 * counterpart in the reference).  Hosts such as an XLA FFI handler, whose
 * framework has reserved the GPU for its own pool, or fixed-budget deployments
 * that forbid allocation after start-up, cannot supply a workspace; this entry
 * point takes it from a static device array of RF_NS_NOALLOC_MAX_WORKSPACE
 * bytes that every GPU loading the library keeps until exit.  Problems whose
 * rf_newton_schulz_workspace_size exceeds that are rejected with RF_EINVAL.
 * All calls on a device share the array (nothing in it needs clearing: each
 * call writes every byte it reads), so calls that overlap on the GPU race:
 * keep them on one stream.  The first call on a device looks the array's
 * address up (cudaGetSymbolAddress) and should come before any stream
 * capture; that address belongs to the context current then (after a
 * cudaDeviceReset, use a new process).  Never calls cudaMalloc / cudaFree. */
#define RF_NS_NOALLOC_MAX_WORKSPACE ((size_t)32 << 20)
rf_status rf_newton_schulz_noalloc(const void* x, int32_t x_dtype, void* out, int32_t out_dtype,
                                   int64_t batch, int64_t rows, int64_t cols, const float* coeffs,
                                   int32_t n_coeff_rows, int32_t ns_steps, float eps, int32_t precision,
                                   void* stream);

/* Deferred tail for gathered orthogonalised leaves (multi-GPU path):
 * out = -lr * (shape_scale * O + decay * p), O read from `o` in leaf layout. */
typedef struct rf_tail_leaf {
  const void* o;      /* [n] orthogonalised leaf, o_dtype */
  const void* param;  /* [n], param_dtype, may be NULL when decay == 0 */
  void* out;          /* [n], out_dtype */
  int64_t n;
  int32_t o_dtype, param_dtype, out_dtype;
  float shape_scale, decay;
  int32_t decay_in_f32;  /* as in rf_muon_leaf */
} rf_tail_leaf;
/* max_ctas_per_sm: 0 = default occupancy; 1-2 leaves room for a persistent
 * Newton-Schulz GEMM CTA on the same SM when this runs beside it. */
rf_status rf_muon_tail(const rf_tail_leaf* leaves, int32_t n_leaves, float lr, int32_t max_ctas_per_sm,
                       void* stream);

/* (N)AdamW fallback leaves (adam.py:123-233 + decay + LR). */
typedef struct rf_adam_leaf {
  const void* grad;   /* [n], grad_dtype */
  float* mu;          /* [n] first moment (state_dtype storage), in place */
  float* nu;          /* [n] second moment (state_dtype storage), in place */
  const void* param;  /* [n], param_dtype; may be NULL when decay == 0 */
  void* out;          /* [n], out_dtype */
  int64_t n;
  int32_t grad_dtype, param_dtype, out_dtype;
  float decay;
  /* dtype the product decay * p is rounded to: the parameter dtype for
   * optax.add_decayed_weights (weakly typed Python float), RF_F32 for the
   * in-transform decay of scale_by_adam (utils.py:79-90). */
  int32_t decay_rounding;
  /* RF_F32, or RF_BF16: both moments stored as bfloat16 with stochastic
   * rounding (adam.py:219-222), noise streams from the two seeds. */
  int32_t state_dtype;
  uint64_t sr_seed_mu, sr_seed_nu;
  /* Optional [n] element-wise decay mask (nonzero byte: decay this element),
   * the array masks of the in-transform decay (utils.py:79-90, 173-197:
   * where(mask, u + wd * p, u)); NULL: every element. */
  const uint8_t* decay_mask;
  /* Magma (adam.py:204-215), as in rf_muon_leaf; needs the workspace of
   * rf_adam_params. */
  float* magma_score;
  int32_t magma_keep;
  int32_t apply_mode;   /* as in rf_muon_leaf (out in param_dtype) */
  uint64_t apply_seed;
} rf_adam_leaf;
typedef struct rf_adam_params {
  /* b1, b2 as the caller's double-precision scalars: the reference forms
   * (1.0 - b2) and (1.0 - b1) from Python floats before the float32 cast
   * (utils.py:486, adam.py:154), but 1 - float32(b1) for the first moment
   * (utils.py:333). */
  double b1, b2;
  float eps, eps_root;
  int32_t count;      /* state.count before this step */
  int32_t nesterov;
  float lr;
  int32_t max_ctas_per_sm;  /* as for rf_muon_tail */
  float magma_tau;
  /* Device workspace for the Magma reductions (sized by
   * rf_adamw_workspace_size; may be NULL / 0 when no leaf uses Magma). */
  void* workspace;
  size_t workspace_bytes;
} rf_adam_params;
rf_status rf_adamw_workspace_size(const rf_adam_leaf* leaves, int32_t n_leaves, size_t* bytes);
rf_status rf_adamw_update(const rf_adam_leaf* leaves, int32_t n_leaves, const rf_adam_params* params,
                          void* stream);

/* Parameter apply p <- p + u (utils.py:648-708): the sum in float32, then
 * the parameter dtype.  bfloat16 parameters round stochastically when
 * `stochastic` (utils.py:342-371: 16 random bits are added below the bf16
 * significand, then truncated; +-Inf and NaN get no noise), else to nearest
 * even; other dtypes round to nearest even.  The random bits are the
 * SplitMix64 sequence seeded with the leaf's `seed` (16 bits per element,
 * in element order); the reference draws them from JAX's Threefry stream, so
 * the two agree in distribution, not bit for bit.  `out` may alias `param`. */
typedef struct rf_apply_leaf {
  const void* param;   /* [n], param_dtype */
  const void* update;  /* [n], update_dtype */
  void* out;           /* [n], param_dtype */
  int64_t n;
  int32_t param_dtype, update_dtype;
  uint64_t seed;
} rf_apply_leaf;
rf_status rf_apply_updates(const rf_apply_leaf* leaves, int32_t n_leaves, int32_t stochastic, void* stream);

/* ------------------------------------------------------------------------
 * Peer transport for the multi-GPU Muon update (one process per GPU, one
 * node).  No reference counterpart: the reference runs every Muon leaf on
 * every device.  The sharded update gathers each owner's orthogonalised
 * leaves by pushing them with the copy engines into the other ranks' buffers
 * (mapped through CUDA IPC), so the gather takes no SMs from the
 * Newton-Schulz GEMMs; cross-rank ordering uses 32-bit epoch flags.
 * ------------------------------------------------------------------------ */
typedef struct rf_ipc_handle {
  unsigned char bytes[64];  /* a cudaIpcMemHandle_t */
} rf_ipc_handle;

/* Handle of the device allocation that contains `ptr` (memory from
 * cudaMalloc, e.g. the PyTorch caching allocator's segments), and the byte
 * offset of `ptr` from the allocation's base. */
rf_status rf_ipc_export(const void* ptr, rf_ipc_handle* handle, size_t* offset);
/* Maps another process's allocation into the current device's context (peer
 * access enabled on demand) and returns its base; the same handle opened
 * twice returns the same base.  Add the exporter's offset. */
rf_status rf_ipc_open(const rf_ipc_handle* handle, void** base);
/* Releases one rf_ipc_open of `base`; the mapping goes with the last. */
rf_status rf_ipc_close(void* base);
/* Stream-ordered copy engine copy of `bytes` between device pointers of
 * this or a mapped peer allocation (no kernel). */
rf_status rf_peer_copy(void* dst, const void* src, size_t bytes, void* stream);
/* After the stream's prior work: a system-scope release store of `value` to
 * each flags[i] (local or mapped peer addresses; n <= 64). */
rf_status rf_flags_signal(uint32_t* const* flags, int32_t n, uint32_t value, void* stream);
/* Blocks the stream until every flags[i] (i != skip, n <= 64, local memory)
 * reaches `target` (wrap-around compare), polling with system-scope acquire
 * loads for at most `timeout_s`; on expiry the wait gives up, the stream moves
 * on and the next rf_sync_check reports RF_ETIMEOUT. */
rf_status rf_flags_wait(const uint32_t* flags, int32_t n, int32_t skip, uint32_t target, double timeout_s,
                        void* stream);

/* Diagnostics. */
const char* rf_last_error(void);
rf_status rf_version(int32_t* major, int32_t* minor, int32_t* patch);
/* Number of kernels this library launched in this process (for bench accounting). */
int64_t rf_kernel_launch_count(void);
/* Launch profiling of the Newton-Schulz GEMM kernel: while enabled, every
 * NS GEMM launch is bracketed by CUDA events on its own stream.
 * rf_profile_end synchronises those events and returns the summed kernel
 * time, the launch count, and the dense algorithmic FLOPs (X X^T: 2m^2n,
 * A A: 2m^3, B X: 2m^2n per matrix) and executed FLOPs (symmetric products
 * visit only tiles that touch the upper triangle) of those launches. */
rf_status rf_profile_begin(void);
rf_status rf_profile_end(double* gemm_ms, int64_t* launches, double* algorithmic_flops,
                         double* executed_flops);
/* Synchronises `stream`, then reports any sticky CUDA error or a bounded
 * device-side wait that gave up (RF_ETIMEOUT) since the last check. */
rf_status rf_sync_check(void* stream);
/* Non-blocking form of rf_sync_check's wait test: after the stream's prior
 * work, copies the two device error words to dst[0] (a bounded wait in the
 * tensor-core kernels gave up) and dst[1] (a cross-rank flag wait gave up);
 * dst is 2 int32 of pinned host or device memory.  A nonzero word means the
 * results of work before it are invalid; rf_sync_check then reports
 * RF_ETIMEOUT and clears the words.  Nothing is cleared here. */
rf_status rf_error_snapshot(int32_t* dst, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ROLLFAST_B200_H_ */

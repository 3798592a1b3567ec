// C-ABI entry points of librollfast_b200 (declared in include/rollfast_b200.h).
//
// Host orchestration of one Muon-branch step:
//   1. momentum + direction sum-of-squares (k_momentum_sumsq), per grad dtype,
//      in launches of <= kMaxLeavesPerLaunch leaves;
//   2. per-matrix Frobenius scale (k_norm_finalize);
//   3. leaves grouped by their NS shape (m <= n after the transpose the
//      reference applies when rows > cols); each group, in sub-batches of at
//      most kMaxLeavesPerLaunch leaves, gets its padded operand X~0
//      (k_ns_load) and ns_steps x {X X^T, bA + cA^2, aX + BX} GEMM stages, the
//      last one writing the update (or O) straight into each leaf.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "rf_kernels.cuh"

namespace rf {

// ---------------------------------------------------------------------------
// Errors and bookkeeping
// ---------------------------------------------------------------------------
static thread_local std::string t_last_error;
static std::atomic<int64_t> g_launches{0};

void set_error(const std::string& msg) { t_last_error = msg; }
rf_status fail(rf_status st, const std::string& msg) {
  set_error(msg);
  return st;
}
rf_status check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RF_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return RF_OK;
}
void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int num_sms() {
  static std::mutex mu;
  static std::map<int, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  cache[dev] = n;
  return n;
}

rf_status take_device_error();  // rf_ns_tc.cu
rf_status take_peer_error();    // rf_peer.cu
rf_status snapshot_device_error(int32_t* dst, cudaStream_t st);  // rf_ns_tc.cu
rf_status snapshot_peer_error(int32_t* dst, cudaStream_t st);    // rf_peer.cu

// ---------------------------------------------------------------------------
// Host-side scalar factors, formed in float32 like the reference.
// ---------------------------------------------------------------------------
static float f32_pow(float b, int e) { return float(std::pow(double(b), double(e))); }

// Programmatic dependent launch of the Newton-Schulz stages (on unless
// ROLLFAST_NS_PDL=0, which launches every stage plainly; results are the same).
static bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("ROLLFAST_NS_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

static MomentumCoeffs momentum_coeffs(const rf_muon_params& p) {
  MomentumCoeffs c{};
  const float beta = p.beta;
  const int t = p.count + 1;  // utils.py:581
  c.beta = beta;
  if (p.accumulator == RF_EMA) {
    c.s = 1.0f - beta;                                                  // utils.py:333
    const int k_mu = p.nesterov ? t + 1 : t;                            // utils.py:590-593
    c.bc_mu = 1.0f - f32_pow(beta, k_mu);                               // utils.py:505
    c.bc_g = 1.0f - f32_pow(beta, t);
    c.mode = p.nesterov ? kDirEmaNesterov : kDirEma;
  } else {
    c.s = 1.0f;                                                         // utils.py:335
    c.bc_mu = c.bc_g = 1.0f;                                            // utils.py:503-504
    c.mode = p.nesterov ? kDirHeavyBallNesterov : kDirHeavyBall;
  }
  c.rbc_mu = float(1.0 / double(c.bc_mu));
  c.rbc_g = float(1.0 / double(c.bc_g));
  return c;
}

// ---------------------------------------------------------------------------
// Plan
// ---------------------------------------------------------------------------
struct LeafPlan {
  int idx;
  const void* g;
  float* mu;
  const void* p;
  void* out;
  int64_t batch, rows, cols, m, n;
  int transposed;
  int gdt, pdt, odt;
  float shape_scale, decay;
  int decay_dt;         // dtype decay * p is rounded to
  int64_t scale_index;  // first matrix in the scale array
  int mu_bf16;          // momentum stored as bfloat16 (stochastic rounding)
  uint64_t sr_seed;
  float* magma_score;   // Magma score (device), null when off
  int magma_keep;
  int apply_mode;       // fused parameter apply (0 off, 1 nearest, 2 stochastic bf16)
  uint64_t apply_seed;
  int64_t magma_chunk;  // first Magma partial-sum chunk of this leaf
};

struct GroupPlan {
  int64_t m, n, mp, np;
  std::vector<std::vector<int>> subs;  // sub-batches of leaf indices (<= kMaxLeavesPerLaunch)
};

struct Plan {
  std::vector<LeafPlan> leaves;
  std::vector<GroupPlan> groups;
  int64_t total_mats = 0;
  int64_t total_chunks = 0;
  size_t off_partials = 0, off_scale = 0, off_ns = 0, bytes = 0;
  size_t off_magma = 0, off_factor = 0;  // Magma partial sums [chunks][3], per-leaf factors
  int64_t magma_chunks = 0;
  size_t ns_bytes = 0;  // one region: max over sub-batches
  int regions = 1;      // 2 when pipelined on an aux stream
  int precision = RF_NS_F16;
};

static size_t ns_elem(int precision) { return precision == RF_NS_F32 ? 4 : 2; }

// Workspace budget of one shape sub-batch (see build_plan).
constexpr size_t kMaxSubBatchBytes = size_t(16) << 30;

static int64_t chunks_per_mat(int64_t numel) { return ceil_div(numel, kChunk); }

static rf_status build_plan(const std::vector<LeafPlan>& in, int precision, Plan& P, int regions = 1) {
  if (precision != RF_NS_F16 && precision != RF_NS_BF16 && precision != RF_NS_F32)
    return fail(RF_EINVAL, "unknown NS precision");
  P.precision = precision;
  P.leaves = in;
  std::map<std::pair<int64_t, int64_t>, int> gindex;
  std::vector<std::vector<int>> members;
  for (size_t i = 0; i < P.leaves.size(); ++i) {
    LeafPlan& L = P.leaves[i];
    if (L.magma_score) {
      L.magma_chunk = P.magma_chunks;
      P.magma_chunks += chunks_per_mat(L.batch * L.rows * L.cols);
    }
    L.scale_index = P.total_mats;
    P.total_mats += L.batch;
    P.total_chunks += L.batch * chunks_per_mat(L.rows * L.cols);
    auto key = std::make_pair(L.m, L.n);
    auto it = gindex.find(key);
    if (it == gindex.end()) {
      gindex[key] = int(members.size());
      members.emplace_back();
      GroupPlan gp;
      gp.m = L.m;
      gp.n = L.n;
      gp.mp = round_up(L.m, 256);
      gp.np = round_up(L.n, 256);
      P.groups.push_back(gp);
      members.back().push_back(int(i));
    } else {
      members[it->second].push_back(int(i));
    }
  }
  const size_t es = ns_elem(precision);
  for (size_t gi = 0; gi < P.groups.size(); ++gi) {
    GroupPlan& gp = P.groups[gi];
    const auto& mem = members[gi];
    // Sub-batches: at most kMaxLeavesPerLaunch leaves, and a workspace region
    // (X0, X1, A~, B~ of every matrix) of about kMaxSubBatchBytes, so that
    // wide groups (e.g. thirty 8192x28672 matrices) leave room in HBM for
    // the state and the updates.
    int64_t mats = 0;
    for (int li : mem) mats += P.leaves[li].batch;
    const double per_mat = double(2 * gp.mp * gp.np + 2 * gp.mp * gp.mp) * double(es);
    const int64_t by_bytes = int64_t(std::ceil(double(mats) * per_mat / double(kMaxSubBatchBytes)));
    const int nsub = int(std::min<int64_t>(int64_t(mem.size()),
                                           std::max(ceil_div(int64_t(mem.size()), kMaxLeavesPerLaunch), by_bytes)));
    const size_t per = (mem.size() + nsub - 1) / nsub;  // even split
    for (size_t s = 0; s < mem.size(); s += per)
      gp.subs.emplace_back(mem.begin() + s, mem.begin() + std::min(mem.size(), s + per));
    for (const auto& sub : gp.subs) {
      int64_t G = 0;
      for (int li : sub) G += P.leaves[li].batch;
      const size_t x = align_up(size_t(G) * gp.mp * gp.np * es, 1024);
      const size_t a = align_up(size_t(G) * gp.mp * gp.mp * es, 1024);
      P.ns_bytes = std::max(P.ns_bytes, 2 * x + 2 * a);
    }
  }
  P.regions = regions;
  P.off_partials = 0;
  P.off_scale = align_up(size_t(P.total_chunks) * 4, 1024);
  P.off_magma = P.off_scale + align_up(size_t(P.total_mats) * 4, 1024);
  P.off_factor = P.off_magma + align_up(size_t(P.magma_chunks) * 12, 1024);
  P.off_ns = P.off_factor + align_up(P.leaves.size() * 4, 1024);
  P.bytes = P.off_ns + size_t(regions) * P.ns_bytes;
  return RF_OK;
}

static rf_status validate_leaf(const rf_muon_leaf& l, int i, bool need_out) {
  const std::string where = "leaf " + std::to_string(i) + ": ";
  if (l.batch <= 0 || l.rows <= 0 || l.cols <= 0) return fail(RF_EINVAL, where + "batch/rows/cols must be positive");
  if (!valid_dtype(l.grad_dtype) || !valid_dtype(l.out_dtype)) return fail(RF_EINVAL, where + "bad dtype");
  if (!l.skip_ns && (!l.grad || !l.mu)) return fail(RF_EINVAL, where + "grad and mu must be non-null");
  if (need_out && !l.out) return fail(RF_EINVAL, where + "out must be non-null");
  if (l.decay != 0.f && (!l.param || !valid_dtype(l.param_dtype)))
    return fail(RF_EINVAL, where + "param (valid dtype) required when decay != 0");
  if (l.mu_dtype != RF_F32 && l.mu_dtype != RF_BF16)
    return fail(RF_EINVAL, where + "mu_dtype must be float32 or bfloat16");
  if (l.apply_mode < 0 || l.apply_mode > 2) return fail(RF_EINVAL, where + "apply_mode must be 0, 1 or 2");
  if (l.apply_mode && (!l.param || l.out_dtype != l.param_dtype))
    return fail(RF_EINVAL, where + "a fused apply needs param, and out in the parameter dtype");
  return RF_OK;
}

// Launches the momentum pass (sum of squares) and the per-matrix norm for
// the leaves `ids` of one sub-batch; `chunk_base` is the first partial-sum
// slot this sub-batch owns.
static rf_status prepare_norms(const Plan& P, const std::vector<int>& ids, const MomentumCoeffs& mc, float* partials,
                               int64_t chunk_base, float* denom, float eps, cudaStream_t st) {
  int64_t cursor = chunk_base;
  for (int gdt : {int(RF_F32), int(RF_BF16), int(RF_F16)}) {
    std::vector<int> sel;
    for (int i : ids)
      if (P.leaves[i].gdt == gdt) sel.push_back(i);
    for (size_t s = 0; s < sel.size(); s += kMaxLeavesPerLaunch) {
      MomentumLaunch L{};
      L.c = mc;
      L.partials = partials + cursor;
      int64_t chunks = 0, mats = 0;
      for (size_t k = s; k < std::min(sel.size(), s + size_t(kMaxLeavesPerLaunch)); ++k) {
        const LeafPlan& lp = P.leaves[sel[k]];
        MomentumLeaf& ml = L.leaf[L.n++];
        ml.g = lp.g;
        ml.mu = lp.mu;
        ml.mu_bf16 = lp.mu_bf16;
        ml.numel = lp.rows * lp.cols;
        ml.chunk_begin = chunks;
        ml.mat_begin = mats;
        ml.scale_index = lp.scale_index;
        ml.chunks_per_mat = int32_t(chunks_per_mat(ml.numel));
        const size_t ge = dtype_size(gdt);
        ml.vec_ok = (ml.numel % 8 == 0) && (reinterpret_cast<uintptr_t>(lp.g) % 16 == 0) &&
                    (!lp.mu || reinterpret_cast<uintptr_t>(lp.mu) % 16 == 0) && ((ml.numel * int64_t(ge)) % 16 == 0);
        chunks += lp.batch * ml.chunks_per_mat;
        mats += lp.batch;
      }
      L.total_chunks = chunks;
      L.total_mats = mats;
      cursor += chunks;
      RF_TRY(launch_momentum_sumsq(L, gdt, st));
      RF_TRY(launch_norm_finalize(L, denom, eps, st));
    }
  }
  return RF_OK;
}

// Magma for the leaves `ids` (magma.py:86-128): partial sums of <g, mu_t>,
// |g|^2, |mu_t|^2 from the previous momentum (so this runs before the
// momentum pass updates it), then each leaf's new score and factor.
static rf_status magma_pass(const Plan& P, const std::vector<int>& ids, const MomentumCoeffs& mc, float tau,
                            uint8_t* base, cudaStream_t st) {
  float* partials = reinterpret_cast<float*>(base + P.off_magma);
  float* factors = reinterpret_cast<float*>(base + P.off_factor);
  std::vector<int> sel;
  for (int i : ids)
    if (P.leaves[i].magma_score) sel.push_back(i);
  for (size_t s0 = 0; s0 < sel.size(); s0 += kMaxLeavesPerLaunch) {
    MagmaDotLaunch D{};
    MagmaFinLaunch F{};
    D.s = mc.s;
    D.beta = mc.beta;
    F.tau = tau;
    const int64_t first = P.leaves[sel[s0]].magma_chunk;
    D.partials = partials + 3 * first;
    F.partials = partials + 3 * first;
    int64_t chunks = 0;
    for (size_t k = s0; k < std::min(sel.size(), s0 + size_t(kMaxLeavesPerLaunch)); ++k) {
      const LeafPlan& lp = P.leaves[sel[k]];
      const int64_t n = lp.batch * lp.rows * lp.cols;
      MagmaDotLeaf& d = D.leaf[D.n++];
      d.g = lp.g;
      d.mu = lp.mu;
      d.n = n;
      d.chunk_begin = chunks;
      d.gdt = lp.gdt;
      d.mu_bf16 = lp.mu_bf16;
      d.vec_ok = (n % 8 == 0) && (reinterpret_cast<uintptr_t>(lp.g) % 16 == 0) &&
                 (reinterpret_cast<uintptr_t>(lp.mu) % 16 == 0);
      MagmaFinLeaf& f = F.leaf[F.n++];
      f.chunk_begin = chunks;
      f.chunks = chunks_per_mat(n);
      f.score = lp.magma_score;
      f.factor = factors + sel[k];
      f.keep = lp.magma_keep;
      chunks += f.chunks;
    }
    D.total_chunks = chunks;
    RF_TRY(launch_magma_dot(D, st));
    RF_TRY(launch_magma_finalize(F, st));
  }
  return RF_OK;
}

// RAII set of events (host objects; no device memory).
struct EventPool {
  std::vector<cudaEvent_t> ev;
  ~EventPool() {
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
  }
  rf_status get(cudaEvent_t* out) {
    cudaEvent_t e;
    cudaError_t err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (err != cudaSuccess) return fail(RF_ECUDA, std::string("cudaEventCreate: ") + cudaGetErrorString(err));
    ev.push_back(e);
    *out = e;
    return RF_OK;
  }
};

// Runs the Muon pipeline for the leaves of `P` (all have NS work), one shape
// sub-batch after another.  Per sub-batch: momentum + norms + operand load
// (HBM-bound, on `aux` when given, else on `st`) and ns_steps x 3 GEMM stages
// on `st`.  With `aux`, sub-batch k+1's preparation overlaps sub-batch k's
// GEMMs; workspace regions alternate, so preparing k+2 waits for k's GEMMs.
static rf_status run_pipeline(const Plan& P, const MomentumCoeffs& mc, const float* coeffs, int n_coeff_rows,
                              int ns_steps, float eps, int precond, int adaptive, int fuse_tail, float lr,
                              int reserve_sms, void* ws, size_t ws_bytes, cudaStream_t st, cudaStream_t aux,
                              float magma_tau = 2.f) {
  if (P.leaves.empty()) return RF_OK;
  if (!ws || ws_bytes < P.bytes)
    return fail(RF_EINVAL, "workspace too small: need " + std::to_string(P.bytes) + " bytes, got " +
                               std::to_string(ws_bytes));
  if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(RF_EINVAL, "workspace must be 256-byte aligned");
  if (aux && P.regions < 2) return fail(RF_EINVAL, "an aux stream needs a workspace sized with pipelined = 1");
  uint8_t* base = static_cast<uint8_t*>(ws);
  float* partials = reinterpret_cast<float*>(base + P.off_partials);
  float* denom = reinterpret_cast<float*>(base + P.off_scale);
  const cudaStream_t prep = aux ? aux : st;
  const size_t es = ns_elem(P.precision);
  EventPool events;
  cudaEvent_t start_ev = nullptr;
  if (aux) {
    // The aux stream starts after everything already queued on `st`.
    RF_TRY(events.get(&start_ev));
    cudaEventRecord(start_ev, st);
    cudaStreamWaitEvent(aux, start_ev, 0);
  }
  std::vector<cudaEvent_t> done;  // per sub-batch: its GEMMs finished (on st)
  int64_t chunk_base = 0;
  int k = 0;
  for (const GroupPlan& gp : P.groups) {
    const NsScales sc = ns_scales(gp.m, P.precision);
    for (const auto& sub : gp.subs) {
      const int region = aux ? (k & 1) : 0;
      uint8_t* ns = base + P.off_ns + size_t(region) * P.ns_bytes;
      int64_t G = 0, sub_chunks = 0;
      for (int li : sub) {
        G += P.leaves[li].batch;
        sub_chunks += P.leaves[li].batch * chunks_per_mat(P.leaves[li].rows * P.leaves[li].cols);
      }
      const size_t xbytes = align_up(size_t(G) * gp.mp * gp.np * es, 1024);
      const size_t abytes = align_up(size_t(G) * gp.mp * gp.mp * es, 1024);
      uint8_t* X0 = ns;
      uint8_t* X1 = ns + xbytes;
      uint8_t* Am = ns + 2 * xbytes;
      uint8_t* Bm = Am + abytes;

      // ---- preparation: momentum, norms, operand load ----
      if (aux && k >= 2) cudaStreamWaitEvent(aux, done[k - 2], 0);  // region reuse
      if (P.magma_chunks) RF_TRY(magma_pass(P, sub, mc, magma_tau, base, prep));
      RF_TRY(prepare_norms(P, sub, mc, partials, chunk_base, denom, eps, prep));
      chunk_base += sub_chunks;

      LoadLaunch ld{};
      ld.c = mc;
      ld.mp = gp.mp;
      ld.np = gp.np;
      ld.denom = denom;
      ld.sx = sc.sx;
      ld.x = X0;
      ld.group_mats = G;
      NsGemmArgs ga{};
      ga.precision = P.precision;
      ga.reserve_sms = reserve_sms;
      ga.G = G;
      ga.m = gp.m;
      ga.n = gp.n;
      ga.mp = gp.mp;
      ga.np = gp.np;
      ga.fuse_tail = fuse_tail;
      ga.neg_lr = -lr;
      ga.out_scale = 1.0f / sc.sx;
      int64_t gm = 0;
      for (int li : sub) {
        const LeafPlan& lp = P.leaves[li];
        LoadLeaf& l = ld.leaf[ld.n++];
        l.mu_bf16 = lp.mu_bf16;
        l.sr_seed = lp.sr_seed;
        // The last operand load stores a bf16 momentum, unless the adaptive
        // pass (which still needs the previous state) runs afterwards.
        l.store_mu = lp.mu_bf16 && !adaptive && precond == RF_PRECOND_FROBENIUS;
        l.g = lp.g;
        l.mu = lp.mu;
        l.rows = lp.rows;
        l.cols = lp.cols;
        l.group_mat_begin = gm;
        l.norm_index = lp.scale_index;
        l.transposed = lp.transposed;
        l.gdt = lp.gdt;
        l.vec_ok = (lp.cols % 8 == 0) && (reinterpret_cast<uintptr_t>(lp.g) % 16 == 0) &&
                   (!lp.mu || reinterpret_cast<uintptr_t>(lp.mu) % 16 == 0);
        FinalLeaf& f = ga.final_leaf[ga.n_final++];
        f.out = lp.out;
        f.p = lp.p;
        f.group_mat_begin = gm;
        f.transposed = lp.transposed;
        f.out_dtype = lp.odt;
        f.p_dtype = lp.pdt;
        f.shape_scale = lp.shape_scale;
        f.decay = lp.decay;
        f.decay_dt = lp.decay_dt;
        f.scale_dev = lp.magma_score ? reinterpret_cast<const float*>(base + P.off_factor) + li : nullptr;
        f.apply_mode = lp.apply_mode;
        f.apply_seed = lp.apply_seed;
        // Runs of 32 along the leaf's rows: length n (NS columns) for a
        // plain leaf, m (NS rows) for a transposed one.
        f.vec_ok = ((lp.transposed ? gp.m : gp.n) % 8 == 0) && (reinterpret_cast<uintptr_t>(lp.out) % 16 == 0) &&
                   (!lp.p || reinterpret_cast<uintptr_t>(lp.p) % 16 == 0);
        gm += lp.batch;
      }
      for (int gdt : {int(RF_F32), int(RF_BF16), int(RF_F16)}) {
        bool any = false;
        for (int li : sub) any |= P.leaves[li].gdt == gdt;
        if (any) RF_TRY(launch_ns_load(ld, gdt, P.precision, prep));
      }
      if (aux) {
        cudaEvent_t ready;
        RF_TRY(events.get(&ready));
        cudaEventRecord(ready, aux);
        cudaStreamWaitEvent(st, ready, 0);
      }

      // ---- preconditioning other than Frobenius (rf_precond.cu) ----
      // A~ of the Frobenius-normalised operand gives the variant's scales
      // (new per-matrix denominators, or per-row factors for aol); the
      // operand is then loaded again with them.  The Lanczos basis lives in
      // Bm and the small scratch in X1, both unused until iteration 1.
      if (precond != RF_PRECOND_FROBENIUS && ns_steps > 0) {
        ga.stage = kSyrkXXt;
        ga.a_op = ga.b_op = X0;
        ga.aux = nullptr;
        ga.out = Am;
        ga.alpha = sc.sa / (sc.sx * sc.sx);
        ga.beta = 0.f;
        RF_TRY(launch_ns_gemm(ga, st));
        int64_t begins[kMaxLeavesPerLaunch], nidx[kMaxLeavesPerLaunch];
        for (int i = 0; i < ld.n; ++i) {
          begins[i] = ld.leaf[i].group_mat_begin;
          nidx[i] = ld.leaf[i].norm_index;
        }
        const float* rows = nullptr;
        RF_TRY(launch_precondition(precond, P.precision, Am, G, gp.m, gp.mp, sc.sa, begins, nidx, ld.n, denom, eps,
                                   Bm, abytes, X1, xbytes, &rows, st));
        ld.row_scale = rows;
        for (int i = 0; i < ld.n; ++i) ld.leaf[i].store_mu = ld.leaf[i].mu_bf16 && !adaptive;
        for (int gdt : {int(RF_F32), int(RF_BF16), int(RF_F16)}) {
          bool any = false;
          for (int li : sub) any |= P.leaves[li].gdt == gdt;
          if (any) RF_TRY(launch_ns_load(ld, gdt, P.precision, st));
        }
      }

      // ---- Newton-Schulz GEMM stages on st ----
      // Every stage but the first directly follows another stage on st and
      // is launched as its programmatic dependent (its prologue overlaps the
      // previous stage's drain); the first follows the operand load and, on
      // the multi-stream path, an event join, and is launched plainly.
      uint8_t* xc = X0;
      uint8_t* xn = X1;
      for (int it = 0; it < ns_steps; ++it) {
        const float* cf = coeffs + 3 * (n_coeff_rows == 0 ? 0 : it);
        const float ca = cf[0], cb = cf[1], cc = cf[2];
        // A~ = (sa / sx^2) X~ X~^T
        ga.pdl = it > 0 && pdl_enabled();
        ga.stage = kSyrkXXt;
        ga.a_op = ga.b_op = xc;
        ga.aux = nullptr;
        ga.out = Am;
        ga.alpha = sc.sa / (sc.sx * sc.sx);
        ga.beta = 0.f;
        RF_TRY(launch_ns_gemm(ga, st));
        // B~ = sb (b A + c A A) = (c sb / sa^2) A~ A~ + (b sb / sa) A~
        ga.pdl = pdl_enabled();
        ga.stage = kSyrkPoly;
        ga.a_op = ga.b_op = ga.aux = Am;
        ga.out = Bm;
        ga.alpha = cc * sc.sb / (sc.sa * sc.sa);
        ga.beta = cb * sc.sb / sc.sa;
        RF_TRY(launch_ns_gemm(ga, st));
        // X~' = sx (a X + B X) = (1 / sb) B~ X~ + a X~
        ga.stage = (it == ns_steps - 1) ? kGemmBXFinal : kGemmBX;
        ga.a_op = Bm;
        ga.b_op = ga.aux = xc;
        ga.out = xn;
        ga.alpha = 1.0f / sc.sb;
        ga.beta = ca;
        RF_TRY(launch_ns_gemm(ga, st));
        std::swap(xc, xn);
      }
      if (aux) {
        cudaEvent_t fin;
        RF_TRY(events.get(&fin));
        cudaEventRecord(fin, st);
        done.push_back(fin);
      }
      ++k;
    }
  }
  return RF_OK;
}

static rf_status leaves_from_abi(const rf_muon_leaf* leaves, int32_t n, std::vector<LeafPlan>& out,
                                 bool need_out) {
  if (n < 0 || (n > 0 && !leaves)) return fail(RF_EINVAL, "null leaf table");
  for (int i = 0; i < n; ++i) {
    const rf_muon_leaf& l = leaves[i];
    RF_TRY(validate_leaf(l, i, need_out));
    if (l.skip_ns) continue;
    LeafPlan p{};
    p.idx = i;
    p.g = l.grad;
    p.mu = l.mu;
    p.p = l.param;
    p.out = l.out;
    p.batch = l.batch;
    p.rows = l.rows;
    p.cols = l.cols;
    p.transposed = l.rows > l.cols;
    p.m = std::min(l.rows, l.cols);
    p.n = std::max(l.rows, l.cols);
    p.gdt = l.grad_dtype;
    p.pdt = l.param ? l.param_dtype : RF_F32;
    p.odt = l.out_dtype;
    p.shape_scale = l.shape_scale;
    p.decay = l.decay;
    p.decay_dt = l.decay_in_f32 ? RF_F32 : p.pdt;
    p.mu_bf16 = l.mu_dtype == RF_BF16;
    p.sr_seed = l.sr_seed;
    p.magma_score = l.magma_score;
    p.magma_keep = l.magma_keep ? 1 : 0;
    p.apply_mode = l.apply_mode;
    p.apply_seed = l.apply_seed;
    out.push_back(p);
  }
  return RF_OK;
}

// Number of NS iterations: a triple repeats ns_steps times, a schedule runs
// all of its rows.
static rf_status check_coeffs(const float* coeffs, int n_rows, int steps, int* iters) {
  if (!coeffs) return fail(RF_EINVAL, "coeffs must be non-null");
  if (n_rows < 0) return fail(RF_EINVAL, "n_coeff_rows must be >= 0");
  if (n_rows == 0 && steps < 1) return fail(RF_EINVAL, "ns_steps must be >= 1");
  *iters = n_rows == 0 ? steps : n_rows;
  return RF_OK;
}

}  // namespace rf

using namespace rf;

extern "C" {

const char* rf_last_error(void) { return t_last_error.c_str(); }

rf_status rf_version(int32_t* major, int32_t* minor, int32_t* patch) {
  if (!major || !minor || !patch) return fail(RF_EINVAL, "null output pointer");
  *major = 0;
  *minor = 1;
  *patch = 0;
  return RF_OK;
}

int64_t rf_kernel_launch_count(void) { return g_launches.load(); }

rf_status rf_sync_check(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(RF_ECUDA, std::string("stream sync: ") + cudaGetErrorString(e));
  RF_TRY(take_peer_error());
  return take_device_error();
}

rf_status rf_error_snapshot(int32_t* dst, void* stream) {
  if (!dst) return fail(RF_EINVAL, "null output pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  RF_TRY(snapshot_device_error(dst, st));
  return snapshot_peer_error(dst + 1, st);
}

rf_status rf_muon_workspace_size(const rf_muon_leaf* leaves, int32_t n_leaves, int32_t precision, int32_t pipelined,
                                 size_t* bytes) {
  if (!bytes) return fail(RF_EINVAL, "null output pointer");
  std::vector<LeafPlan> lp;
  RF_TRY(leaves_from_abi(leaves, n_leaves, lp, false));
  Plan P;
  RF_TRY(build_plan(lp, precision, P, pipelined ? 2 : 1));
  *bytes = P.bytes;
  return RF_OK;
}

// adaptive (muon.py:272-282) after an unfused pipeline: `out` holds O; each
// leaf's <d, O> goes to ip[] (the per-matrix scale slots, free once the NS
// stages are queued), then out <- -lr (shape <d,O> O + decay p) in place, or
// out <- <d,O> O without the tail.  Partial sums reuse the momentum partials.
static rf_status adaptive_pass(const Plan& P, const MomentumCoeffs& mc, int fuse_tail, float lr, void* ws,
                               cudaStream_t st) {
  uint8_t* base = static_cast<uint8_t*>(ws);
  float* partials = reinterpret_cast<float*>(base + P.off_partials);
  float* ip = reinterpret_cast<float*>(base + P.off_scale);
  int64_t chunk_base = 0;
  const int nl = int(P.leaves.size());
  for (int s0 = 0; s0 < nl; s0 += kMaxLeavesPerLaunch) {
    AdaptiveLaunch A{};
    A.c = mc;
    A.partials = partials + chunk_base;
    TailLaunch T{};
    T.neg_lr = fuse_tail ? -lr : 1.f;
    int64_t chunks = 0;
    for (int i = s0; i < std::min(nl, s0 + kMaxLeavesPerLaunch); ++i) {
      const LeafPlan& lp = P.leaves[i];
      const int64_t n = lp.batch * lp.rows * lp.cols;
      AdaptiveLeaf& a = A.leaf[A.n++];
      a.g = lp.g;
      a.mu = lp.mu;
      a.mu_bf16 = lp.mu_bf16;
      a.sr_seed = lp.sr_seed;
      a.o = lp.out;
      a.n = n;
      a.chunk_begin = chunks;
      a.gdt = lp.gdt;
      a.odt = lp.odt;
      TailLeafDev& t = T.leaf[T.n++];
      t.o = lp.out;
      t.p = fuse_tail ? lp.p : nullptr;
      t.out = lp.out;
      t.n = n;
      t.chunk_begin = chunks;
      t.odt = t.outdt = lp.odt;
      t.pdt = lp.p ? lp.pdt : RF_F32;
      t.shape_scale = fuse_tail ? lp.shape_scale : 1.f;
      t.decay = fuse_tail ? lp.decay : 0.f;
      t.decay_dt = lp.decay_dt;
      t.dev_scale = ip + i;
      t.vec_ok = (n % 8 == 0) && (reinterpret_cast<uintptr_t>(lp.out) % 16 == 0) &&
                 (!t.p || reinterpret_cast<uintptr_t>(lp.p) % 16 == 0);
      chunks += ceil_div(n, kChunk);
    }
    A.total_chunks = T.total_chunks = chunks;
    for (int gdt : {int(RF_F32), int(RF_BF16), int(RF_F16)}) {
      bool any = false;
      for (int k = 0; k < A.n; ++k) any |= A.leaf[k].gdt == gdt;
      if (any) RF_TRY(launch_adaptive_dot(A, gdt, st));
    }
    RF_TRY(launch_adaptive_finalize(A, ip + s0, st));
    RF_TRY(launch_tail(T, st));
    chunk_base += chunks;
  }
  return RF_OK;
}

rf_status rf_muon_update(const rf_muon_leaf* leaves, int32_t n_leaves, const rf_muon_params* params,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!params) return fail(RF_EINVAL, "null params");
  const rf_muon_params& p = *params;
  if (!(p.beta >= 0.f && p.beta < 1.f)) return fail(RF_EINVAL, "beta must be in [0, 1)");
  if (!(p.eps > 0.f)) return fail(RF_EINVAL, "eps must be positive");
  if (p.accumulator != RF_EMA && p.accumulator != RF_HEAVY_BALL)
    return fail(RF_EINVAL, "momentum_accumulator must be 'ema' or 'heavy_ball'");
  if (p.count < 0) return fail(RF_EINVAL, "count must be >= 0");
  int iters = 0;
  RF_TRY(check_coeffs(p.coeffs, p.n_coeff_rows, p.ns_steps, &iters));
  if (p.reserve_sms < 0) return fail(RF_EINVAL, "reserve_sms must be >= 0");
  std::vector<LeafPlan> lp;
  RF_TRY(leaves_from_abi(leaves, n_leaves, lp, true));
  Plan P;
  RF_TRY(build_plan(lp, p.precision, P, p.aux_stream ? 2 : 1));
  if (p.preconditioning < RF_PRECOND_FROBENIUS || p.preconditioning > RF_PRECOND_SCHATTEN)
    return fail(RF_EINVAL, "unknown preconditioning");
  for (const LeafPlan& l : P.leaves)
    if (l.apply_mode && (!p.fuse_tail || p.adaptive))
      return fail(RF_ENOTSUP, "a fused apply needs fuse_tail = 1 and adaptive = 0");
  if (P.magma_chunks) {
    if (!(p.magma_tau > 0.f)) return fail(RF_EINVAL, "magma_tau must be positive");
    if (p.adaptive) return fail(RF_ENOTSUP, "Magma together with adaptive is not supported");
    if (!p.fuse_tail) return fail(RF_ENOTSUP, "Magma needs the fused tail (fuse_tail = 1)");
  }
  if (p.adaptive) {
    const MomentumCoeffs mc = momentum_coeffs(p);
    RF_TRY(run_pipeline(P, mc, p.coeffs, p.n_coeff_rows, iters, p.eps, p.preconditioning, 1, 0, 0.f, p.reserve_sms,
                        workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                        static_cast<cudaStream_t>(p.aux_stream)));
    return adaptive_pass(P, mc, p.fuse_tail, p.lr, workspace, static_cast<cudaStream_t>(stream));
  }
  return run_pipeline(P, momentum_coeffs(p), p.coeffs, p.n_coeff_rows, iters, p.eps, p.preconditioning, 0,
                      p.fuse_tail, p.lr,
                      p.reserve_sms, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                      static_cast<cudaStream_t>(p.aux_stream), p.magma_tau);
}

rf_status rf_muon_direction(const rf_muon_leaf* leaves, int32_t n_leaves, const rf_muon_params* params,
                            void* stream) {
  if (!params) return fail(RF_EINVAL, "null params");
  const rf_muon_params& p = *params;
  if (!(p.beta >= 0.f && p.beta < 1.f)) return fail(RF_EINVAL, "beta must be in [0, 1)");
  if (p.accumulator != RF_EMA && p.accumulator != RF_HEAVY_BALL)
    return fail(RF_EINVAL, "momentum_accumulator must be 'ema' or 'heavy_ball'");
  if (n_leaves < 0 || (n_leaves > 0 && !leaves)) return fail(RF_EINVAL, "null leaf table");
  const MomentumCoeffs mc = momentum_coeffs(p);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DirLaunch D{};
  D.c = mc;
  int64_t chunks = 0;
  for (int i = 0; i < n_leaves; ++i) {
    const rf_muon_leaf& l = leaves[i];
    RF_TRY(validate_leaf(l, i, true));
    if (l.skip_ns) continue;
    if (l.out_dtype != RF_F32) return fail(RF_EINVAL, "direction output must be float32");
    DirLeafDev& d = D.leaf[D.n++];
    d.g = l.grad;
    d.mu = l.mu;
    d.out = static_cast<float*>(l.out);
    d.n = l.batch * l.rows * l.cols;
    d.chunk_begin = chunks;
    d.gdt = l.grad_dtype;
    d.mu_bf16 = l.mu_dtype == RF_BF16;
    d.sr_seed = l.sr_seed;
    chunks += ceil_div(d.n, kChunk);
    if (D.n == kMaxLeavesPerLaunch) {
      D.total_chunks = chunks;
      RF_TRY(launch_direction(D, st));
      D = DirLaunch{};
      D.c = mc;
      chunks = 0;
    }
  }
  D.total_chunks = chunks;
  if (D.n) RF_TRY(launch_direction(D, st));
  return RF_OK;
}

static rf_status ns_plan(int64_t batch, int64_t rows, int64_t cols, int32_t precision, Plan& P, const void* x,
                         int32_t x_dtype, void* out, int32_t out_dtype) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return fail(RF_EINVAL, "batch/rows/cols must be positive");
  LeafPlan l{};
  l.g = x;
  l.mu = nullptr;
  l.out = out;
  l.batch = batch;
  l.rows = rows;
  l.cols = cols;
  l.transposed = rows > cols;
  l.m = std::min(rows, cols);
  l.n = std::max(rows, cols);
  l.gdt = x_dtype;
  l.pdt = RF_F32;
  l.odt = out_dtype;
  l.shape_scale = 1.f;
  l.decay = 0.f;
  l.decay_dt = RF_F32;
  return build_plan({l}, precision, P);
}

rf_status rf_newton_schulz_workspace_size(int64_t batch, int64_t rows, int64_t cols, int32_t precision,
                                          size_t* bytes) {
  if (!bytes) return fail(RF_EINVAL, "null output pointer");
  Plan P;
  RF_TRY(ns_plan(batch, rows, cols, precision, P, nullptr, RF_F32, nullptr, RF_F32));
  *bytes = P.bytes;
  return RF_OK;
}

rf_status rf_newton_schulz(const void* x, int32_t x_dtype, void* out, int32_t out_dtype, int64_t batch,
                           int64_t rows, int64_t cols, const float* coeffs, int32_t n_coeff_rows, int32_t ns_steps,
                           float eps, int32_t preconditioning, int32_t precision, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!x || !out) return fail(RF_EINVAL, "x and out must be non-null");
  if (preconditioning < RF_PRECOND_FROBENIUS || preconditioning > RF_PRECOND_SCHATTEN)
    return fail(RF_EINVAL, "unknown preconditioning");
  if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype)) return fail(RF_EINVAL, "bad dtype");
  if (!(eps > 0.f)) return fail(RF_EINVAL, "eps must be positive");
  int iters = 0;
  RF_TRY(check_coeffs(coeffs, n_coeff_rows, ns_steps, &iters));
  Plan P;
  RF_TRY(ns_plan(batch, rows, cols, precision, P, x, x_dtype, out, out_dtype));
  MomentumCoeffs mc{};
  mc.mode = kDirIdentity;
  return run_pipeline(P, mc, coeffs, n_coeff_rows, iters, eps, preconditioning, 0, 0, 0.f, 0, workspace, workspace_bytes,
                      static_cast<cudaStream_t>(stream), nullptr);
}

rf_status rf_apply_updates(const rf_apply_leaf* leaves, int32_t n_leaves, int32_t stochastic, void* stream) {
  if (n_leaves < 0 || (n_leaves > 0 && !leaves)) return fail(RF_EINVAL, "null leaf table");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int s = 0; s < n_leaves; s += kMaxLeavesPerLaunch) {
    ApplyLaunch A{};
    A.stochastic = stochastic ? 1 : 0;
    int64_t chunks = 0;
    for (int i = s; i < std::min(n_leaves, s + kMaxLeavesPerLaunch); ++i) {
      const rf_apply_leaf& l = leaves[i];
      const std::string where = "apply leaf " + std::to_string(i) + ": ";
      if (l.n < 0 || (l.n > 0 && (!l.param || !l.update || !l.out))) return fail(RF_EINVAL, where + "bad pointers");
      if (!valid_dtype(l.param_dtype) || !valid_dtype(l.update_dtype)) return fail(RF_EINVAL, where + "bad dtype");
      ApplyLeafDev& d = A.leaf[A.n++];
      d.p = l.param;
      d.u = l.update;
      d.out = l.out;
      d.n = l.n;
      d.chunk_begin = chunks;
      d.pdt = l.param_dtype;
      d.udt = l.update_dtype;
      d.seed = l.seed;
      d.vec_ok = (l.n % 8 == 0) && (reinterpret_cast<uintptr_t>(l.param) % 16 == 0) &&
                 (reinterpret_cast<uintptr_t>(l.update) % 16 == 0) && (reinterpret_cast<uintptr_t>(l.out) % 16 == 0);
      chunks += ceil_div(l.n, kChunk);
    }
    A.total_chunks = chunks;
    RF_TRY(launch_apply(A, st));
  }
  return RF_OK;
}

rf_status rf_muon_tail(const rf_tail_leaf* leaves, int32_t n_leaves, float lr, int32_t max_ctas_per_sm,
                       void* stream) {
  if (n_leaves < 0 || (n_leaves > 0 && !leaves)) return fail(RF_EINVAL, "null leaf table");
  if (max_ctas_per_sm < 0) return fail(RF_EINVAL, "max_ctas_per_sm must be >= 0");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int s = 0; s < n_leaves; s += kMaxLeavesPerLaunch) {
    TailLaunch T{};
    T.neg_lr = -lr;
    T.max_ctas_per_sm = max_ctas_per_sm;
    int64_t chunks = 0;
    for (int i = s; i < std::min(n_leaves, s + kMaxLeavesPerLaunch); ++i) {
      const rf_tail_leaf& l = leaves[i];
      if (l.n < 0 || (l.n > 0 && (!l.o || !l.out))) return fail(RF_EINVAL, "tail leaf " + std::to_string(i) + ": bad pointers");
      if (!valid_dtype(l.o_dtype) || !valid_dtype(l.out_dtype)) return fail(RF_EINVAL, "tail leaf: bad dtype");
      if (l.decay != 0.f && (!l.param || !valid_dtype(l.param_dtype)))
        return fail(RF_EINVAL, "tail leaf: param required when decay != 0");
      TailLeafDev& d = T.leaf[T.n++];
      d.o = l.o;
      d.p = l.param;
      d.out = l.out;
      d.n = l.n;
      d.chunk_begin = chunks;
      d.odt = l.o_dtype;
      d.pdt = l.param ? l.param_dtype : RF_F32;
      d.outdt = l.out_dtype;
      d.shape_scale = l.shape_scale;
      d.decay = l.decay;
      d.decay_dt = l.decay_in_f32 ? RF_F32 : d.pdt;
      d.vec_ok = (l.n % 8 == 0) && (reinterpret_cast<uintptr_t>(l.o) % 16 == 0) &&
                 (reinterpret_cast<uintptr_t>(l.out) % 16 == 0) &&
                 (!l.param || reinterpret_cast<uintptr_t>(l.param) % 16 == 0);
      chunks += ceil_div(l.n, kChunk);
    }
    T.total_chunks = chunks;
    RF_TRY(launch_tail(T, st));
  }
  return RF_OK;
}

// Magma workspace of rf_adamw_update: [chunks][3] partial sums, then one
// factor per leaf.
static void adam_magma_layout(const rf_adam_leaf* leaves, int32_t n, int64_t* chunks, size_t* off_factor,
                              size_t* bytes) {
  int64_t c = 0;
  for (int i = 0; i < n; ++i)
    if (leaves[i].magma_score) c += ceil_div(leaves[i].n, kChunk);
  *chunks = c;
  *off_factor = align_up(size_t(c) * 12, 256);
  *bytes = c ? *off_factor + align_up(size_t(n) * 4, 256) : 0;
}

rf_status rf_adamw_workspace_size(const rf_adam_leaf* leaves, int32_t n_leaves, size_t* bytes) {
  if (!bytes) return fail(RF_EINVAL, "null output pointer");
  if (n_leaves < 0 || (n_leaves > 0 && !leaves)) return fail(RF_EINVAL, "null leaf table");
  int64_t chunks = 0;
  size_t off = 0;
  adam_magma_layout(leaves, n_leaves, &chunks, &off, bytes);
  return RF_OK;
}

rf_status rf_adamw_update(const rf_adam_leaf* leaves, int32_t n_leaves, const rf_adam_params* params,
                          void* stream) {
  if (!params) return fail(RF_EINVAL, "null params");
  if (n_leaves < 0 || (n_leaves > 0 && !leaves)) return fail(RF_EINVAL, "null leaf table");
  const rf_adam_params& p = *params;
  int64_t magma_chunks = 0;
  size_t off_factor = 0, magma_bytes = 0;
  adam_magma_layout(leaves, n_leaves, &magma_chunks, &off_factor, &magma_bytes);
  if (magma_chunks) {
    if (!(p.magma_tau > 0.f)) return fail(RF_EINVAL, "magma_tau must be positive");
    if (!p.workspace || p.workspace_bytes < magma_bytes)
      return fail(RF_EINVAL, "Magma needs a workspace of " + std::to_string(magma_bytes) + " bytes");
  }
  if (p.count < 0) return fail(RF_EINVAL, "count must be >= 0");
  if (p.max_ctas_per_sm < 0) return fail(RF_EINVAL, "max_ctas_per_sm must be >= 0");
  AdamCoeffs c{};
  const int t = p.count + 1;
  const float b1f = float(p.b1), b2f = float(p.b2);
  c.b1 = b1f;
  c.b2 = b2f;
  c.one_minus_b1 = 1.0f - b1f;                 // utils.py:333 (1 - decay32)
  c.one_minus_b2 = float(1.0 - p.b2);          // utils.py:486 ((1.0 - decay) with a Python float)
  c.one_minus_b1_py = float(1.0 - p.b1);       // adam.py:154 ((1.0 - b1) with a Python float)
  c.bc1 = 1.0f - f32_pow(b1f, t);              // adam.py:137
  c.bc1_next = 1.0f - f32_pow(b1f, t + 1);     // adam.py:141
  c.bc2 = 1.0f - f32_pow(b2f, t);              // adam.py:138
  c.eps = p.eps;
  c.eps_root = p.eps_root;
  c.neg_lr = -p.lr;
  c.nesterov = p.nesterov;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* magma_partials = magma_chunks ? static_cast<float*>(p.workspace) : nullptr;
  float* factors = magma_chunks ? reinterpret_cast<float*>(static_cast<uint8_t*>(p.workspace) + off_factor) : nullptr;
  if (magma_chunks) {
    // Scores and factors first (they read the previous first moment, which
    // the AdamW kernel then updates in place): adam.py:204-215 with
    // mu_t = (1 - b1) g + b1 mu.
    std::vector<int> sel;
    for (int i = 0; i < n_leaves; ++i)
      if (leaves[i].magma_score) sel.push_back(i);
    int64_t cursor = 0;
    for (size_t s0 = 0; s0 < sel.size(); s0 += kMaxLeavesPerLaunch) {
      MagmaDotLaunch D{};
      MagmaFinLaunch F{};
      D.s = c.one_minus_b1;
      D.beta = c.b1;
      D.partials = magma_partials + 3 * cursor;
      F.partials = D.partials;
      F.tau = p.magma_tau;
      int64_t chunks = 0;
      for (size_t k = s0; k < std::min(sel.size(), s0 + size_t(kMaxLeavesPerLaunch)); ++k) {
        const rf_adam_leaf& l = leaves[sel[k]];
        if (l.n > 0 && (!l.grad || !l.mu)) return fail(RF_EINVAL, "adam leaf: bad pointers");
        MagmaDotLeaf& d = D.leaf[D.n++];
        d.g = l.grad;
        d.mu = l.mu;
        d.n = l.n;
        d.chunk_begin = chunks;
        d.gdt = l.grad_dtype;
        d.mu_bf16 = l.state_dtype == RF_BF16;
        d.vec_ok = (l.n % 8 == 0) && (reinterpret_cast<uintptr_t>(l.grad) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(l.mu) % 16 == 0);
        MagmaFinLeaf& f = F.leaf[F.n++];
        f.chunk_begin = chunks;
        f.chunks = ceil_div(l.n, kChunk);
        f.score = l.magma_score;
        f.factor = factors + sel[k];
        f.keep = l.magma_keep ? 1 : 0;
        chunks += f.chunks;
      }
      D.total_chunks = chunks;
      cursor += chunks;
      RF_TRY(launch_magma_dot(D, st));
      RF_TRY(launch_magma_finalize(F, st));
    }
  }
  for (int s = 0; s < n_leaves; s += kMaxLeavesPerLaunch) {
    AdamLaunch A{};
    A.c = c;
    A.max_ctas_per_sm = p.max_ctas_per_sm;
    int64_t chunks = 0;
    for (int i = s; i < std::min(n_leaves, s + kMaxLeavesPerLaunch); ++i) {
      const rf_adam_leaf& l = leaves[i];
      if (l.n < 0 || (l.n > 0 && (!l.grad || !l.mu || !l.nu || !l.out)))
        return fail(RF_EINVAL, "adam leaf " + std::to_string(i) + ": bad pointers");
      if (!valid_dtype(l.grad_dtype) || !valid_dtype(l.out_dtype)) return fail(RF_EINVAL, "adam leaf: bad dtype");
      if (l.decay != 0.f && (!l.param || !valid_dtype(l.param_dtype)))
        return fail(RF_EINVAL, "adam leaf: param required when decay != 0");
      AdamLeafDev& d = A.leaf[A.n++];
      d.g = l.grad;
      d.mu = l.mu;
      d.nu = l.nu;
      d.p = l.param;
      d.out = l.out;
      d.n = l.n;
      d.chunk_begin = chunks;
      d.gdt = l.grad_dtype;
      d.pdt = l.param ? l.param_dtype : RF_F32;
      d.odt = l.out_dtype;
      d.decay = l.decay;
      d.decay_dt = l.decay_rounding;
      if (l.state_dtype != RF_F32 && l.state_dtype != RF_BF16)
        return fail(RF_EINVAL, "adam leaf: state_dtype must be float32 or bfloat16");
      d.sdt = l.state_dtype;
      d.seed_mu = l.sr_seed_mu;
      d.seed_nu = l.sr_seed_nu;
      d.mask = l.decay != 0.f ? l.decay_mask : nullptr;
      if (l.apply_mode < 0 || l.apply_mode > 2) return fail(RF_EINVAL, "adam leaf: apply_mode must be 0, 1 or 2");
      if (l.apply_mode && (!l.param || l.out_dtype != l.param_dtype))
        return fail(RF_EINVAL, "adam leaf: a fused apply needs param, and out in the parameter dtype");
      d.apply_mode = l.apply_mode;
      d.apply_seed = l.apply_seed;
      d.scale_dev = l.magma_score ? factors + i : nullptr;
      d.vec_ok = (l.n % 8 == 0) && (reinterpret_cast<uintptr_t>(l.grad) % 16 == 0) &&
                 (reinterpret_cast<uintptr_t>(l.mu) % 16 == 0) && (reinterpret_cast<uintptr_t>(l.nu) % 16 == 0) &&
                 (reinterpret_cast<uintptr_t>(l.out) % 16 == 0) &&
                 (!l.param || reinterpret_cast<uintptr_t>(l.param) % 16 == 0) &&
                 (!d.mask || reinterpret_cast<uintptr_t>(d.mask) % 8 == 0);
      if (l.decay != 0.f && !valid_dtype(l.decay_rounding)) return fail(RF_EINVAL, "adam leaf: bad decay_rounding");
      chunks += ceil_div(l.n, kChunk);
    }
    A.total_chunks = chunks;
    RF_TRY(launch_adamw(A, st));
  }
  return RF_OK;
}

}  // extern "C"

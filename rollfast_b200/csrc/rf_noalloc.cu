// rf_newton_schulz_noalloc: the orthogonalize_fn entry point for callers that
// cannot allocate device memory.
//
// Some hosts give a custom operation no way to allocate: an XLA FFI handler
// runs inside a framework that has already reserved most of the GPU for its
// own pool and only hands out the buffers it planned, and embedded or
// fixed-budget deployments forbid allocation after start-up.  Such callers
// cannot provide the workspace rf_newton_schulz asks for.  This variant takes
// its workspace from a file-scope device array instead, so the caller passes
// only inputs, outputs and a stream.
//
// Limits and sharing:
//   * The array holds kStaticScratchBytes (32 MiB).  Every GPU that loads this
//     library keeps that much memory reserved until the process exits.
//   * Problems whose workspace (rf_newton_schulz_workspace_size) exceeds it
//     are rejected with RF_EINVAL; with 16-bit operands that admits, e.g., a
//     1024 x 4096 matrix, or 8 matrices of 512 x 1024.
//   * All calls on a device share the one array and it keeps the last call's
//     contents.  Every byte a call reads is first written by that same call,
//     so nothing has to be cleared; but two calls whose work overlaps on the
//     GPU (e.g. issued on different streams) race on the array.  Order them on
//     one stream.
//   * The device address of the array is looked up once per device with
//     cudaGetSymbolAddress, by the first call made with that device current;
//     make that first call before any stream capture.  The address belongs to
//     the CUDA context current at that call: after a cudaDeviceReset, or
//     from another context on the same device, use a new process.
// The computation is the one rf_newton_schulz performs (same kernels).
#include <mutex>

#include "rf_kernels.cuh"

// The scratch itself.  In host code `g_ns_scratch` names a host-side stand-in,
// not device memory: only the address obtained from cudaGetSymbolAddress may
// be handed to kernels.
static __device__ __align__(256) unsigned char g_ns_scratch[RF_NS_NOALLOC_MAX_WORKSPACE];

namespace {

constexpr size_t kStaticScratchBytes = RF_NS_NOALLOC_MAX_WORKSPACE;
constexpr int kMaxDevices = 64;

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

rf_status scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return rf::fail(RF_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return rf::fail(RF_EINVAL, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ns_scratch);
    if (e != cudaSuccess || !p)
      return rf::fail(RF_ECUDA, std::string("cudaGetSymbolAddress(static NS scratch): ") + cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return RF_OK;
}

}  // namespace

extern "C" rf_status rf_newton_schulz_noalloc(const void* x, int32_t x_dtype, void* out, int32_t out_dtype,
                                             int64_t batch, int64_t rows, int64_t cols, const float* coeffs,
                                             int32_t n_coeff_rows, int32_t ns_steps, float eps, int32_t precision,
                                             void* stream) {
  size_t need = 0;
  RF_TRY(rf_newton_schulz_workspace_size(batch, rows, cols, precision, &need));
  if (need > kStaticScratchBytes)
    return rf::fail(RF_EINVAL, "rf_newton_schulz_noalloc: this problem needs " + std::to_string(need) +
                                   " bytes of workspace, more than the " + std::to_string(kStaticScratchBytes) +
                                   "-byte static scratch; use rf_newton_schulz with a caller workspace");
  void* ws = nullptr;
  RF_TRY(scratch_for_current_device(&ws));
  return rf_newton_schulz(x, x_dtype, out, out_dtype, batch, rows, cols, coeffs, n_coeff_rows, ns_steps, eps,
                          RF_PRECOND_FROBENIUS, precision, ws, kStaticScratchBytes, stream);
}

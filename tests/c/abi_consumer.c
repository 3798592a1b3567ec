/* A plain C consumer of librollfast_b200.so: what a rollfast maintainer's
 * FFI shim links against.  Exercises the entry points that need no GPU
 * (version, workspace planning, argument validation) and prints one line per
 * check; tests/test_c_abi_cpu.py compiles and runs it. */
#include <stdio.h>
#include <string.h>

#include "rollfast_b200.h"

static int failures = 0;

static void check(int cond, const char* what) {
  printf("%s %s\n", cond ? "ok" : "FAIL", what);
  if (!cond) ++failures;
}

int main(void) {
  int32_t a = -1, b = -1, c = -1;
  check(rf_version(&a, &b, &c) == RF_OK && a == 0 && b >= 1, "rf_version");

  /* Llama-3-8B-like leaves: q (4096x4096) and down (14336x4096, transposed). */
  rf_muon_leaf leaves[2];
  memset(leaves, 0, sizeof(leaves));
  static float dummy[8];
  for (int i = 0; i < 2; ++i) {
    leaves[i].grad = dummy;
    leaves[i].mu = dummy;
    leaves[i].out = dummy;
    leaves[i].batch = 1;
    leaves[i].grad_dtype = RF_BF16;
    leaves[i].out_dtype = RF_F32;
    leaves[i].mu_dtype = RF_F32;
  }
  leaves[0].rows = 4096; leaves[0].cols = 4096;
  leaves[1].rows = 14336; leaves[1].cols = 4096;
  size_t ws16 = 0, ws32 = 0, ws_pipe = 0;
  check(rf_muon_workspace_size(leaves, 2, RF_NS_F16, 0, &ws16) == RF_OK && ws16 > 0, "workspace f16");
  check(rf_muon_workspace_size(leaves, 2, RF_NS_F32, 0, &ws32) == RF_OK && ws32 > ws16, "workspace f32 > f16");
  check(rf_muon_workspace_size(leaves, 2, RF_NS_F16, 1, &ws_pipe) == RF_OK && ws_pipe > ws16,
        "pipelined workspace holds two regions");
  size_t nsw = 0;
  check(rf_newton_schulz_workspace_size(8, 1024, 4096, RF_NS_F16, &nsw) == RF_OK && nsw > 0, "NS workspace");

  /* Contracts: bad arguments return RF_EINVAL with a message, never abort. */
  check(rf_muon_update(leaves, 2, NULL, NULL, 0, NULL) == RF_EINVAL && strlen(rf_last_error()) > 0,
        "null params -> RF_EINVAL");
  leaves[1].mu_dtype = 7;
  check(rf_muon_workspace_size(leaves, 2, RF_NS_F16, 0, &ws16) == RF_EINVAL, "bad mu_dtype -> RF_EINVAL");
  leaves[1].mu_dtype = RF_F32;
  leaves[0].rows = 0;
  check(rf_muon_workspace_size(leaves, 2, RF_NS_F16, 0, &ws16) == RF_EINVAL, "empty leaf -> RF_EINVAL");
  check(rf_muon_workspace_size(leaves, 2, 9, 0, &ws16) == RF_EINVAL, "bad precision -> RF_EINVAL");
  check(rf_flags_wait(NULL, 65, 0, 1, 1.0, NULL) == RF_EINVAL, "flag wait n > 64 -> RF_EINVAL");
  check(rf_ipc_export(NULL, NULL, NULL) == RF_EINVAL, "ipc export null -> RF_EINVAL");
  check(rf_apply_updates(NULL, 0, 0, NULL) == RF_OK, "apply with no leaves is a no-op");
  check(rf_kernel_launch_count() == 0, "no kernel launched");

  printf("%d failures\n", failures);
  return failures != 0;
}

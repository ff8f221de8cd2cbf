// Library-wide entry points: version string and the thread-local last-error message that every
// failing entry point fills before returning a nonzero status.
#include <stdarg.h>
#include <stdio.h>
#include <mutex>
#include <vector>

#include "oa_common.cuh"
#include "../../include/openattention_b200.h"

static thread_local char g_err[1024] = "";

int oa_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int oa_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return OA_OK;
}

namespace {
struct SmemOptIn {
  const void* kernel;
  int device;
  size_t static_bytes;  // the kernel's static shared memory
  size_t dyn_set;       // the dynamic limit set so far (0: the 48 KB default)
  bool carveout_set;    // the largest shared-memory carveout was requested
};
std::mutex g_smem_mu;
std::vector<SmemOptIn> g_smem;
}  // namespace

// The kernel's static size is queried once per device and the limit is raised only when a launch
// needs more than was set before: both are host calls that are not free, and launches in a decode
// loop repeat the same sizes.
int oa_smem_opt_in(const void* kernel, size_t dyn, const char* what, bool max_carveout) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_smem_mu);
  SmemOptIn* ent = nullptr;
  for (SmemOptIn& x : g_smem)
    if (x.kernel == kernel && x.device == dev) ent = &x;
  if (ent == nullptr) {
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    g_smem.push_back(SmemOptIn{kernel, dev, fa.sharedSizeBytes, 0, false});
    ent = &g_smem.back();
  }
  if (dyn + ent->static_bytes > 48 * 1024 && dyn > ent->dyn_set) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    ent->dyn_set = dyn;
  }
  if (max_carveout && !ent->carveout_set) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    ent->carveout_set = true;
  }
  return OA_OK;
}

extern "C" const char* oa_version(void) { return "openattention_b200 0.1.0 (sm_100a)"; }

extern "C" const char* oa_last_error_string(void) { return g_err; }

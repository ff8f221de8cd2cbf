// Library-wide entry points: version string and the thread-local last-error message that every
// failing entry point fills before returning a nonzero status.
#include <stdarg.h>
#include <stdio.h>

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

int oa_smem_opt_in(const void* kernel, size_t dyn, const char* what) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  if (dyn + fa.sharedSizeBytes > 48 * 1024) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    if (e != cudaSuccess) return oa_fail(OA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  return OA_OK;
}

extern "C" const char* oa_version(void) { return "openattention_b200 0.1.0 (sm_100a)"; }

extern "C" const char* oa_last_error_string(void) { return g_err; }

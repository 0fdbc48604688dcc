// C-ABI plumbing: error strings, version, device queries, workspace status.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace mv {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MV_OK;
  return fail(MV_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

}  // namespace mv

extern "C" int mv_version(void) { return 100; }  // 0.1.0

extern "C" const char* mv_last_error(void) { return mv::g_err; }

extern "C" int mv_workspace_status(void* workspace, int clear, unsigned int* code, unsigned int* info,
                                   void* stream) {
  if (workspace == nullptr) return mv::fail(MV_ERR_INVALID, "mv_workspace_status: null workspace");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int h[3] = {0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(h, workspace, sizeof(h), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return mv::cuda_status(e, "mv_workspace_status");
  if (code) *code = h[1];
  if (info) *info = h[2];
  if (clear && (h[1] || h[2])) {
    e = cudaMemsetAsync(static_cast<char*>(workspace) + 4, 0, 8, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return mv::cuda_status(e, "mv_workspace_status(clear)");
  }
  return MV_OK;
}

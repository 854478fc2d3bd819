// Error plumbing and diagnostics of the C ABI.

#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace lbx {

static thread_local char t_err[512] = {0};

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return LBX_OK;
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return LBX_ECUDA;
}

}  // namespace lbx

extern "C" int lbx_last_error(char *buf, size_t n) {
  if (!buf || n == 0) return LBX_EINVAL;
  strncpy(buf, lbx::t_err, n - 1);
  buf[n - 1] = 0;
  return LBX_OK;
}

extern "C" int lbx_device_error(int32_t *out_host, cudaStream_t stream) {
  if (!out_host) return LBX_EINVAL;
  cudaError_t e = cudaMemcpyFromSymbolAsync(out_host, lbx::g_lbx_device_error, sizeof(int32_t), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  return lbx::cuda_status(e, "read device error word");
}

extern "C" int lbx_clear_device_error(cudaStream_t stream) {
  static const int32_t zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(lbx::g_lbx_device_error, &zero, sizeof(int32_t), 0,
                                          cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  return lbx::cuda_status(e, "clear device error word");
}

extern "C" const char *lbx_version(void) { return "lbx 0.1 sm_100a"; }

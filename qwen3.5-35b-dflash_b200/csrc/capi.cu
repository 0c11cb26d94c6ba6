// Status and error-message plumbing of the C ABI.
#include <cstdarg>
#include <cstdio>

#include "qw_common.cuh"

namespace qw {

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t err, const char* what) {
  set_error("%s: CUDA error %d (%s)", what, static_cast<int>(err), cudaGetErrorString(err));
  return QW_ERR_CUDA;
}

}  // namespace qw

extern "C" int qw_abi_version(void) { return QW_ABI_VERSION; }

extern "C" const char* qw_last_error(void) { return qw::g_error; }

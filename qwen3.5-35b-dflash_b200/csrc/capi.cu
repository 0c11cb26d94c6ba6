// Status and error-message plumbing of the C ABI.
#include <atomic>
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

static std::atomic<long long> g_inject_limit{0};
static std::atomic<unsigned> g_inject_excess{0};

WaitInjection wait_injection() { return WaitInjection{g_inject_limit.load(), g_inject_excess.load()}; }

// Reports the sticky words of the linear and MoE waits as one status and clears them.
__global__ void wait_status_kernel(int32_t* lin, int32_t* moe, int32_t* dst, int clear) {
  pdl_wait();   // every kernel before this one has finished (and written its word)
  pdl_trigger();
  if (threadIdx.x == 0) {
    const int s = (*lin != 0 || *moe != 0) ? QW_ERR_TIMEOUT : QW_OK;
    *dst = s;
    if (clear) {
      *lin = 0;
      *moe = 0;
    }
  }
}

static int status_words(int32_t** lin, int32_t** moe) {
  int rc = linear_wait_status_addr(lin);
  if (rc != QW_OK) return rc;
  return moe_wait_status_addr(moe);
}

}  // namespace qw

using namespace qw;

extern "C" int qw_wait_status(int32_t* status, int clear, void* stream) {
  QW_CHECK_ARG(status, "wait_status: null pointer");
  int32_t *lin = nullptr, *moe = nullptr;
  const int rc = status_words(&lin, &moe);
  if (rc != QW_OK) return rc;
  QW_LAUNCH_PDL("wait_status", wait_status_kernel, dim3(1), dim3(32), 0, as_stream(stream), lin, moe, status,
                clear);
  return QW_OK;
}

extern "C" int qw_check_wait_status(int clear, void* stream) {
  int32_t *lin = nullptr, *moe = nullptr;
  int rc = status_words(&lin, &moe);
  if (rc != QW_OK) return rc;
  cudaStream_t st = as_stream(stream);
  cudaError_t err = cudaStreamSynchronize(st);
  if (err != cudaSuccess) return cuda_status(err, "check_wait_status: stream synchronize");
  int32_t h[2] = {0, 0};
  err = cudaMemcpy(&h[0], lin, 4, cudaMemcpyDeviceToHost);
  if (err == cudaSuccess) err = cudaMemcpy(&h[1], moe, 4, cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return cuda_status(err, "check_wait_status: read");
  if (clear && (h[0] || h[1])) {
    err = cudaMemsetAsync(lin, 0, 4, st);
    if (err == cudaSuccess) err = cudaMemsetAsync(moe, 0, 4, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess) return cuda_status(err, "check_wait_status: clear");
  }
  if (h[0] || h[1])
    return fail(QW_ERR_TIMEOUT, "a bounded device wait expired in %s%s%s: the outputs of those launches are "
                "incomplete", h[0] ? "a cluster linear kernel" : "", h[0] && h[1] ? " and " : "",
                h[1] ? "a MoE expert kernel" : "");
  return QW_OK;
}

extern "C" int qw_debug_inject_wait_timeout(int64_t limit_cycles, int64_t tx_excess_bytes) {
  QW_CHECK_ARG(limit_cycles >= 0 && tx_excess_bytes >= 0 && tx_excess_bytes < (1 << 20),
               "inject_wait_timeout: limit >= 0 and 0 <= excess < 2^20 required");
  g_inject_limit.store(limit_cycles);
  g_inject_excess.store(static_cast<unsigned>(tx_excess_bytes));
  return QW_OK;
}

extern "C" int qw_abi_version(void) { return QW_ABI_VERSION; }

extern "C" const char* qw_last_error(void) { return g_error; }

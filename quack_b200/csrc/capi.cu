// Error reporting, version and launch accounting of the C ABI.
#include "qk_common.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>

static thread_local char g_last_error[512] = "";
static std::atomic<long long> g_launches{0};

int qk_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int qk_check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return QK_OK;
  return qk_fail(QK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void qk_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

extern "C" int qk_version(void) { return 100; }
extern "C" const char* qk_last_error(void) { return g_last_error; }
extern "C" long long qk_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

// qk_gemm_blockscaled_noalloc: the block-scaled GEMM for callers that cannot allocate device
// memory.
//
// The regular entry point needs two pieces of scratch memory from its caller: the 4-int status
// block every launch writes to when a bounded wait gives up, and (optionally) 16 int64 of
// per-role cycle counters per launched CTA.  Some callers have nothing to give: a serving
// process that fixed its device-memory plan at start-up and may not call cudaMalloc once it is
// live, or a thin binding from another language that can pass along the pointers it was handed
// but owns no CUDA allocator.  For them the scratch lives here, in a file-scope device array
// that every GPU loading the library holds until the process exits:
//
//     256 bytes (status block) + QK_NOALLOC_MAX_CTAS x 128 bytes (counters) = 33 024 bytes.
//
// Consequences the caller has to know about:
//   * one array per GPU, shared by every call: two calls that overlap on the GPU (different
//     streams, or different host threads) race on the status block and the counters.  Serialise
//     them, or use the regular entry point with one scratch buffer per stream;
//   * the array keeps the previous call's contents; the parts a launch relies on being zero
//     (the status block, the counters when they are requested) are cleared on the stream
//     before every launch;
//   * a launch may use at most QK_NOALLOC_MAX_CTAS CTAs; devices with more SMs, or an explicit
//     `max_ctas` beyond that, are rejected with QK_ERR_TOO_LARGE;
//   * the first call on a device looks up the device address of the array
//     (cudaGetSymbolAddress, with that device current).  Make that first call outside any
//     stream capture.
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include "gemm_host.h"

#include <cstring>
#include <mutex>

namespace {

constexpr int kStatusBytes = 256;
constexpr int kProfBytesPerCta = 16 * 8;
constexpr size_t kScratchBytes = kStatusBytes + static_cast<size_t>(QK_NOALLOC_MAX_CTAS) * kProfBytesPerCta;

// In host code this name is only a handle for cudaGetSymbolAddress, never an address to pass to
// a kernel.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_for_current_device(unsigned char** out, int* sm_count) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return qk_fail(QK_ERR_CUDA, "qk_gemm_blockscaled_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return qk_fail(QK_ERR_UNSUPPORTED, "qk_gemm_blockscaled_noalloc: device index %d", dev);
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return qk_fail(QK_ERR_CUDA, "qk_gemm_blockscaled_noalloc: cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
  *sm_count = sms;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return qk_fail(QK_ERR_CUDA, "qk_gemm_blockscaled_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_ptr[dev];
  return QK_OK;
}

}  // namespace

extern "C" int qk_gemm_blockscaled_noalloc(const qk_gemm_args* args, int* status_out, long long* prof_out) {
  if (args == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled_noalloc: null argument block");
  if (args->status != nullptr || args->prof != nullptr)
    return qk_fail(QK_ERR_INVALID_ARG,
                   "qk_gemm_blockscaled_noalloc: leave args->status and args->prof NULL (the library supplies them); "
                   "pass status_out / prof_out to receive copies");
  if (args->scheduler != QK_SCHED_STATIC)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_gemm_blockscaled_noalloc: static scheduler only (the scratch is sized per persistent CTA)");
  if (args->max_ctas > QK_NOALLOC_MAX_CTAS)
    return qk_fail(QK_ERR_TOO_LARGE, "qk_gemm_blockscaled_noalloc: max_ctas %d exceeds the %d CTAs the static scratch covers",
                   args->max_ctas, QK_NOALLOC_MAX_CTAS);
  unsigned char* scratch = nullptr;
  int sms = 0;
  int rc = scratch_for_current_device(&scratch, &sms);
  if (rc != QK_OK) return rc;
  const int ctas = args->max_ctas > 0 ? (args->max_ctas < sms ? args->max_ctas : sms) : sms;
  if (ctas > QK_NOALLOC_MAX_CTAS)
    return qk_fail(QK_ERR_TOO_LARGE,
                   "qk_gemm_blockscaled_noalloc: this device would launch %d CTAs, the static scratch covers %d; "
                   "set max_ctas or use qk_gemm_blockscaled with your own scratch",
                   ctas, QK_NOALLOC_MAX_CTAS);
  cudaStream_t st = static_cast<cudaStream_t>(args->stream);
  // the array still holds whatever the previous call left: clear what this launch reads as zero
  const size_t clear = prof_out != nullptr ? kScratchBytes : static_cast<size_t>(kStatusBytes);
  cudaError_t e = cudaMemsetAsync(scratch, 0, clear, st);
  if (e != cudaSuccess) return qk_fail(QK_ERR_CUDA, "qk_gemm_blockscaled_noalloc: cudaMemsetAsync: %s", cudaGetErrorString(e));
  qk_gemm_args local;
  std::memcpy(&local, args, sizeof(local));
  local.status = reinterpret_cast<int*>(scratch);
  local.prof = prof_out != nullptr ? reinterpret_cast<long long*>(scratch + kStatusBytes) : nullptr;
  local.max_ctas = ctas;
  rc = qk_gemm_blockscaled(&local);
  if (rc != QK_OK) return rc;
  if (status_out != nullptr) {
    e = cudaMemcpyAsync(status_out, scratch, 4 * sizeof(int), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return qk_fail(QK_ERR_CUDA, "qk_gemm_blockscaled_noalloc: status copy: %s", cudaGetErrorString(e));
  }
  if (prof_out != nullptr) {
    e = cudaMemcpyAsync(prof_out, scratch + kStatusBytes, static_cast<size_t>(QK_NOALLOC_MAX_CTAS) * kProfBytesPerCta,
                        cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return qk_fail(QK_ERR_CUDA, "qk_gemm_blockscaled_noalloc: counter copy: %s", cudaGetErrorString(e));
  }
  return QK_OK;
}

// Peer-memory plumbing of the copy-engine all-gather transport: export / open CUDA IPC handles,
// enqueue device-to-device copies and stream-ordered 32-bit waits and writes.  None of these
// launches a kernel, so none of them needs an SM while a persistent GEMM owns the GPU.
#include "qk_common.h"
#include "../../include/quack_b200.h"

#include <cuda.h>

#include <cstring>
#include <mutex>

namespace {

typedef CUresult (*WaitValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
typedef CUresult (*WriteValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

struct DriverFns {
  WaitValue32Fn wait32 = nullptr;
  WriteValue32Fn write32 = nullptr;
  AddressRangeFn range = nullptr;
};

void* entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return p;
}

const DriverFns& driver() {
  static DriverFns fns;
  static std::once_flag once;
  std::call_once(once, [] {
    fns.wait32 = reinterpret_cast<WaitValue32Fn>(entry("cuStreamWaitValue32"));
    fns.write32 = reinterpret_cast<WriteValue32Fn>(entry("cuStreamWriteValue32"));
    fns.range = reinterpret_cast<AddressRangeFn>(entry("cuMemGetAddressRange"));
  });
  return fns;
}

int cuda_fail(const char* what, cudaError_t e) {
  cudaGetLastError();
  return qk_fail(QK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

static_assert(sizeof(cudaIpcMemHandle_t) == QK_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int qk_ipc_export(const void* ptr, void* handle_out, unsigned long long* offset_out) {
  if (!ptr || !handle_out || !offset_out) return qk_fail(QK_ERR_INVALID_ARG, "qk_ipc_export: null argument");
  const DriverFns& d = driver();
  if (!d.range) return qk_fail(QK_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = d.range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return qk_fail(QK_ERR_CUDA, "cuMemGetAddressRange failed (%d): not a device allocation?", (int)r);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail("cudaIpcGetMemHandle (memory must come from cudaMalloc, not a virtual-memory pool)", e);
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<unsigned long long>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return QK_OK;
}

extern "C" int qk_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return qk_fail(QK_ERR_INVALID_ARG, "qk_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail("cudaIpcOpenMemHandle", e);
  *base_out = p;
  return QK_OK;
}

extern "C" int qk_ipc_close(void* base) {
  if (!base) return QK_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail("cudaIpcCloseMemHandle", e);
  return QK_OK;
}

extern "C" int qk_copy_async(void* dst, const void* src, unsigned long long bytes, void* stream) {
  if (bytes == 0) return QK_OK;
  if (!dst || !src) return qk_fail(QK_ERR_INVALID_ARG, "qk_copy_async: null pointer");
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("cudaMemcpyAsync", e);
  return QK_OK;
}

extern "C" int qk_stream_wait_geq32(void* stream, const void* addr, unsigned int value) {
  if (!addr) return qk_fail(QK_ERR_INVALID_ARG, "qk_stream_wait_geq32: null address");
  if (reinterpret_cast<uintptr_t>(addr) & 3) return qk_fail(QK_ERR_INVALID_ARG, "qk_stream_wait_geq32: address not 4-byte aligned");
  const DriverFns& d = driver();
  if (!d.wait32) return qk_fail(QK_ERR_CUDA, "cuStreamWaitValue32 is not available from the driver");
  const CUresult r = d.wait32(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(addr), value, CU_STREAM_WAIT_VALUE_GEQ);
  if (r != CUDA_SUCCESS) return qk_fail(QK_ERR_CUDA, "cuStreamWaitValue32 failed (%d)", (int)r);
  return QK_OK;
}

extern "C" int qk_stream_write32(void* stream, void* addr, unsigned int value) {
  if (!addr) return qk_fail(QK_ERR_INVALID_ARG, "qk_stream_write32: null address");
  if (reinterpret_cast<uintptr_t>(addr) & 3) return qk_fail(QK_ERR_INVALID_ARG, "qk_stream_write32: address not 4-byte aligned");
  const DriverFns& d = driver();
  if (!d.write32) return qk_fail(QK_ERR_CUDA, "cuStreamWriteValue32 is not available from the driver");
  const CUresult r = d.write32(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(addr), value, CU_STREAM_WRITE_VALUE_DEFAULT);
  if (r != CUDA_SUCCESS) return qk_fail(QK_ERR_CUDA, "cuStreamWriteValue32 failed (%d)", (int)r);
  return QK_OK;
}

extern "C" int qk_stream_ops(const qk_stream_op* ops, int count) {
  if (count < 0 || (count > 0 && ops == nullptr)) return qk_fail(QK_ERR_INVALID_ARG, "qk_stream_ops: bad op list");
  for (int i = 0; i < count; ++i) {
    const qk_stream_op& o = ops[i];
    int rc;
    switch (o.kind) {
      case QK_OP_COPY: rc = qk_copy_async(o.dst, o.src, o.bytes, o.stream); break;
      case QK_OP_WAIT_GEQ32: rc = qk_stream_wait_geq32(o.stream, o.dst, o.value); break;
      case QK_OP_WRITE32: rc = qk_stream_write32(o.stream, o.dst, o.value); break;
      default: return qk_fail(QK_ERR_INVALID_ARG, "qk_stream_ops: op %d has unknown kind %d", i, o.kind);
    }
    if (rc != QK_OK) return rc;
  }
  return QK_OK;
}

// ABI version and status strings of libkvc_b200.so.
#include "kvc_common.cuh"

extern "C" int kvc_abi_version(void) { return KVC_ABI_VERSION; }

extern "C" const char* kvc_status_string(int status) {
  switch (status) {
    case KVC_OK: return "ok";
    case KVC_EINVAL: return "invalid size, count or enum argument";
    case KVC_ENULL: return "required pointer is NULL";
    case KVC_EALIGN: return "pointer or stride misaligned for the kernel";
    case KVC_EUNSUPPORTED: return "geometry not supported by the compiled kernels";
    case KVC_ECUDA: return "CUDA launch failed";
    case KVC_ECAPACITY: return "request exceeds the library's fixed static scratch capacity";
    default: return "unknown status";
  }
}

// Host helpers for callers that already hold raw handles (one call each, no
// framework round trip): an event record and an async copy between any two
// addresses the runtime knows (pinned host or device), both on `stream`.
extern "C" int kvc_record_event(void* event, void* stream) {
  if (!event) return KVC_ENULL;
  if (cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream) != cudaSuccess) {
    cudaGetLastError();
    return KVC_ECUDA;
  }
  return KVC_OK;
}

extern "C" int kvc_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (!dst || !src) return KVC_ENULL;
  if (bytes < 0) return KVC_EINVAL;
  if (bytes == 0) return KVC_OK;
  if (cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, (cudaStream_t)stream) != cudaSuccess) {
    cudaGetLastError();
    return KVC_ECUDA;
  }
  return KVC_OK;
}

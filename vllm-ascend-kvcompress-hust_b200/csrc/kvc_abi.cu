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

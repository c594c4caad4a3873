// Shared device/host helpers for the sm_100a TriAttention kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "kvc.h"

namespace kvc {

constexpr int kBlock = 128;  // tokens per kernel cache block (page)

#define KVC_CHECK_ARG(cond, code) \
  do {                            \
    if (!(cond)) return (code);   \
  } while (0)

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? KVC_OK : KVC_ECUDA;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

// ---- element conversion --------------------------------------------------

struct Bf16 {};
struct Fp16 {};

// Two packed 16-bit elements of one 32-bit word -> floats (low half first).
__device__ __forceinline__ float2 unpack2(uint32_t w, Bf16) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float2 unpack2(uint32_t w, Fp16) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}
__device__ __forceinline__ float unpack1(uint16_t v, Bf16) { return __uint_as_float(uint32_t(v) << 16); }
__device__ __forceinline__ float unpack1(uint16_t v, Fp16) {
  return __half2float(*reinterpret_cast<__half*>(&v));
}

__device__ __forceinline__ uint16_t pack1(float x, Bf16) {
  const __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<const uint16_t*>(&b);
}
__device__ __forceinline__ uint16_t pack1(float x, Fp16) {
  const __half h = __float2half_rn(x);
  return *reinterpret_cast<const uint16_t*>(&h);
}

// Element j (0..7) of a 16-byte vector of 16-bit elements.
template <int J, class E>
__device__ __forceinline__ float elem8(const uint4& v, E e) {
  const uint32_t w = J < 2 ? v.x : J < 4 ? v.y : J < 6 ? v.z : v.w;
  return (J & 1) ? unpack2(w, e).y : unpack2(w, e).x;
}

// 16-byte read-only load that does not allocate in L1 (streamed once).
__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// NaN-propagating max with torch.maximum / amax semantics.
__device__ __forceinline__ float nan_max(float a, float b) {
  return (a != a) ? a : ((b != b || b > a) ? b : a);
}

// torch.nan_to_num(nan=-inf, posinf=1e30, neginf=-inf)
__device__ __forceinline__ float finalize_score(float v) {
  if (v != v) return -INFINITY;
  if (v == INFINITY) return 1e30f;
  return v;
}

// Request owning page p: largest r with page_off[r] <= p (page_off has R+1 entries).
__device__ __forceinline__ int request_of_page(const int32_t* __restrict__ page_off, int R, int p) {
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(page_off + mid) <= p) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void raise_flag(int32_t* flag, int bit) {
  if (flag) atomicOr(flag, bit);
}

// ---- programmatic dependent launch ---------------------------------------
//
// The kernels of a compression step run back to back on one stream.  Each
// starts with pdl_wait() -- before touching any global memory -- which returns
// once the preceding kernel on the stream has completed and its writes are
// visible (and at once when the kernel was launched without the attribute),
// then calls pdl_trigger(), which lets the next kernel be launched while this
// one still runs.  launch_dep() launches with programmatic stream
// serialization, so the next kernel's CTAs are resident and waiting when this
// one ends instead of being launched after it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... Params, typename... Args>
inline void launch_dep(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace kvc

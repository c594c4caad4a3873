// Tensor-parallel score sync over NVLink peer memory (sm_100a).
//
// Every TP rank holds the per-layer head-max rows of its own KV heads,
// rows[l][tok] (the normalisation output), in a buffer the other ranks have
// mapped through CUDA IPC.  One kernel per rank then replaces the MAX
// all-reduce and the layer reduction that follows it:
//
//   1. signal "rows ready" to every rank, wait for every rank's signal;
//   2. for the token range this rank owns (1/world of the step's tokens, in
//      4-token vectors),
//      load every rank's rows over NVLink, take the max over ranks per layer
//      (NaN-propagating, as the TP=1 head max), reduce the layers (sequential
//      fp32 sum / L or max) and finalise exactly as kvc_aggregate_rows does;
//   3. store the finished scores into every rank's agg buffer (plain peer
//      stores), fence, and let the last CTA signal "agg pushed".
//
// A one-warp kernel behind it waits for every rank's "agg pushed" signal, so
// the selection launched next on the stream reads complete scores.  Bytes over
// NVLink per rank: (world-1)/world of the rows (reduce) plus (world-1)/world of
// agg (broadcast), against 2(world-1)/world of the rows for a ring all-reduce.
//
// Flags are per-step epochs (monotonic, never reset), so no clearing pass is
// needed.  Every wait is bounded (2 s of %globaltimer); on expiry the kernel
// raises KVC_DEV_TIMEOUT in the error flag and completes.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "kvc_common.cuh"

namespace kvc {

constexpr uint64_t kTpWaitNs = 2000000000ull;

struct TpArgs {
  const float* const* rows;  // [world] each rank's rows[L][tok_total]
  float* const* agg;         // [world] each rank's agg[tok_total]
  int32_t* const* flags;     // [world] each rank's flags: ready[world], pushed[world], counter
  const int32_t* tokens;
  const int32_t* page_off;
  int32_t* error_flag;
  int64_t tok_total;
  int world, rank, L, R, layer_agg;
  int32_t epoch;
};

__device__ __forceinline__ uint64_t tp_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until flags[0..n) have all reached `epoch`; false when the bound expires.
__device__ bool wait_epochs(const int32_t* flags, int n, int32_t epoch) {
  const uint64_t t0 = tp_now_ns();
  for (int j = 0; j < n; ++j) {
    unsigned it = 0;
    while ((int32_t)((uint32_t)ld_acquire_sys(flags + j) - (uint32_t)epoch) < 0) {
      if ((++it & 127) == 0 && tp_now_ns() - t0 > kTpWaitNs) return false;
      __nanosleep(100);
    }
  }
  return true;
}

__device__ __forceinline__ float4 nan_max4(float4 a, float4 b) {
  return make_float4(nan_max(a.x, b.x), nan_max(a.y, b.y), nan_max(a.z, b.z), nan_max(a.w, b.w));
}

// W: the world size when it is compiled in (1, 2, 4, 8), else 0 (runtime, loads in groups of 8).
// Each thread owns 4 consecutive tokens (one float4; 4 | 128, so they share a page):
// per layer it issues the loads of every rank's row before reducing, so a
// warp keeps W x 16 bytes per lane in flight over NVLink.
template <int W>
__global__ void __launch_bounds__(256) tp_reduce_push_kernel(const __grid_constant__ TpArgs a) {
  __shared__ int ok;
  __shared__ const float* rows_s[KVC_TP_MAX_WORLD];
  __shared__ float* agg_s[KVC_TP_MAX_WORLD];
  const int world = W ? W : a.world;
  for (int p = threadIdx.x; p < world; p += blockDim.x) {
    rows_s[p] = a.rows[p];
    agg_s[p] = a.agg[p];
  }
  int32_t* mine = a.flags[a.rank];
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();  // this rank's rows (previous kernel) before "rows ready"
      for (int p = 0; p < world; ++p) st_release_sys(a.flags[p] + a.rank, a.epoch);
    }
    ok = wait_epochs(mine, world, a.epoch);
    if (!ok) raise_flag(a.error_flag, KVC_DEV_TIMEOUT);
  }
  __syncthreads();
  if (ok) {
    const int64_t quads = a.tok_total >> 2;
    const int64_t per = (quads + world - 1) / world;
    const int64_t lo = (int64_t)a.rank * per;
    const int64_t hi = min64(lo + per, quads);
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t q = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < hi; q += step) {
      const int64_t tok = q << 2;
      const int r = request_of_page(a.page_off, a.R, (int)(tok >> 7));
      const int t = (int)(tok - (int64_t)__ldg(a.page_off + r) * kBlock);
      const int n = __ldg(a.tokens + r);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);  // page padding, as kvc_aggregate_rows
      if (t < n) {
        float4 acc = v;
        for (int l = 0; l < a.L; ++l) {
          const int64_t i = (int64_t)l * a.tok_total + tok;
          float4 m = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
          if constexpr (W > 0) {
            float4 x[W];
#pragma unroll
            for (int p = 0; p < W; ++p) x[p] = *reinterpret_cast<const float4*>(rows_s[p] + i);
#pragma unroll
            for (int p = 0; p < W; ++p) m = nan_max4(m, x[p]);
          } else {
            for (int p0 = 0; p0 < world; p0 += 8) {
              float4 x[8];
#pragma unroll
              for (int k = 0; k < 8; ++k)
                if (p0 + k < world) x[k] = *reinterpret_cast<const float4*>(rows_s[p0 + k] + i);
#pragma unroll
              for (int k = 0; k < 8; ++k)
                if (p0 + k < world) m = nan_max4(m, x[k]);
            }
          }
          if (l == 0) {
            acc = m;
          } else if (a.layer_agg == KVC_AGG_MEAN) {
            acc = make_float4(acc.x + m.x, acc.y + m.y, acc.z + m.z, acc.w + m.w);
          } else {
            acc = nan_max4(acc, m);
          }
        }
        if (a.layer_agg == KVC_AGG_MEAN) {
          const float d = (float)a.L;
          acc = make_float4(__fdiv_rn(acc.x, d), __fdiv_rn(acc.y, d), __fdiv_rn(acc.z, d), __fdiv_rn(acc.w, d));
        }
        v = make_float4(t + 0 < n ? finalize_score(acc.x) : 0.f, t + 1 < n ? finalize_score(acc.y) : 0.f,
                        t + 2 < n ? finalize_score(acc.z) : 0.f, t + 3 < n ? finalize_score(acc.w) : 0.f);
      }
      for (int p = 0; p < world; ++p) *reinterpret_cast<float4*>(agg_s[p] + tok) = v;
    }
  }
  __threadfence_system();  // this thread's peer stores before the completion count
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t* counter = mine + 2 * world;
    if (atomicAdd(counter, 1) == (int)gridDim.x - 1) {
      atomicExch(counter, 0);
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(a.flags[p] + world + a.rank, a.epoch);
    }
  }
}

__global__ void tp_wait_pushed_kernel(const __grid_constant__ TpArgs a) {
  if (threadIdx.x == 0 && !wait_epochs(a.flags[a.rank] + a.world, a.world, a.epoch))
    raise_flag(a.error_flag, KVC_DEV_TIMEOUT);
}

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }
  return fn;
}

}  // namespace kvc

using namespace kvc;

extern "C" int kvc_tp_exchange_flag_words(int world) { return world > 0 ? 2 * world + 1 : 0; }

extern "C" int kvc_tp_exchange_max(const float* const* peer_rows, float* const* peer_agg, int32_t* const* peer_flags,
                                   int world, int rank, int num_layers, int total_pages, const int32_t* tokens,
                                   const int32_t* page_off, int num_requests, int layer_aggregation, int32_t epoch,
                                   int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(peer_rows && peer_agg && peer_flags && tokens && page_off, KVC_ENULL);
  KVC_CHECK_ARG(world >= 1 && world <= KVC_TP_MAX_WORLD && rank >= 0 && rank < world, KVC_EINVAL);
  KVC_CHECK_ARG(num_layers > 0 && total_pages >= 0 && num_requests >= 0 && epoch > 0, KVC_EINVAL);
  KVC_CHECK_ARG(layer_aggregation == KVC_AGG_MEAN || layer_aggregation == KVC_AGG_MAX, KVC_EINVAL);
  TpArgs a{};
  a.rows = peer_rows;
  a.agg = peer_agg;
  a.flags = peer_flags;
  a.tokens = tokens;
  a.page_off = page_off;
  a.error_flag = error_flag;
  a.tok_total = (int64_t)total_pages * kBlock;
  a.world = world;
  a.rank = rank;
  a.L = num_layers;
  a.R = num_requests;
  a.layer_agg = layer_aggregation;
  a.epoch = epoch;
  // every rank runs both kernels every step, even with no tokens, so the
  // epochs of all ranks advance together
  const int64_t quads = a.tok_total / 4;
  const int64_t want = ((quads + world - 1) / world + 255) / 256;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sm_count() * 8));
  cudaStream_t st = (cudaStream_t)stream;
  switch (world) {
    case 1: tp_reduce_push_kernel<1><<<grid, 256, 0, st>>>(a); break;
    case 2: tp_reduce_push_kernel<2><<<grid, 256, 0, st>>>(a); break;
    case 4: tp_reduce_push_kernel<4><<<grid, 256, 0, st>>>(a); break;
    case 8: tp_reduce_push_kernel<8><<<grid, 256, 0, st>>>(a); break;
    default: tp_reduce_push_kernel<0><<<grid, 256, 0, st>>>(a); break;
  }
  int rc = launch_status();
  if (rc != KVC_OK) return rc;
  tp_wait_pushed_kernel<<<1, 32, 0, st>>>(a);
  return launch_status();
}

extern "C" int kvc_ipc_export(int device, const void* ptr, void* handle_out, int64_t* offset_out) {
  KVC_CHECK_ARG(ptr && handle_out && offset_out, KVC_ENULL);
  static_assert(sizeof(cudaIpcMemHandle_t) == KVC_IPC_HANDLE_BYTES, "IPC handle size");
  if (cudaSetDevice(device) != cudaSuccess) return KVC_ECUDA;
  PFN_cuMemGetAddressRange_v3020 range = address_range_fn();
  if (!range) return KVC_EUNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return KVC_ECUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, (void*)base) != cudaSuccess) return KVC_ECUDA;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)((CUdeviceptr)ptr - base);
  return KVC_OK;
}

extern "C" int kvc_ipc_open(int device, const void* handle, void** base_out) {
  KVC_CHECK_ARG(handle && base_out, KVC_ENULL);
  if (cudaSetDevice(device) != cudaSuccess) return KVC_ECUDA;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return KVC_ECUDA;
  }
  *base_out = p;
  return KVC_OK;
}

extern "C" int kvc_ipc_close(int device, void* base) {
  KVC_CHECK_ARG(base, KVC_ENULL);
  if (cudaSetDevice(device) != cudaSuccess) return KVC_ECUDA;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    cudaGetLastError();
    return KVC_ECUDA;
  }
  return KVC_OK;
}

extern "C" int kvc_can_access_peer(int device, int peer) {
  int ok = 0;
  if (device == peer) return 1;
  if (cudaDeviceCanAccessPeer(&ok, device, peer) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return ok;
}

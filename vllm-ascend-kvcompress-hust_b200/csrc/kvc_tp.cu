// Tensor-parallel score sync over NVLink peer memory (sm_100a).
//
// Every TP rank holds the per-layer head-max rows of its own KV heads,
// rows[l][tok] (the normalisation output), in a buffer the other ranks have
// mapped through CUDA IPC.  One kernel per rank replaces the MAX all-reduce
// and the layer reduction that follows it:
//
//   1. the first CTA to start signals "rows ready" to every rank (the rows are
//      complete: the previous kernel on the stream wrote them); every CTA waits
//      for every rank's signal;
//   2. the rank owns 1/world of the step's tokens, in 4-token quads.  A CTA
//      takes a group of Q quads with L/ceil(L/64) threads per quad, so each
//      thread loads one (quad, layer) from every rank over NVLink (all loads of
//      a group in flight at once) and keeps their NaN-propagating max in
//      shared memory; one thread per quad then reduces the layers in order
//      (sequential fp32 sum / L, or max) and finalises exactly as
//      kvc_aggregate_rows does;
//   3. the CTA stores the finished quads into every rank's agg buffer (plain
//      peer stores, consecutive threads on consecutive quads), fences, and the
//      last CTA signals "agg pushed" to every rank, then waits for every rank's
//      "agg pushed" before the kernel ends, so the selection launched next on
//      the stream reads complete scores and no rank is still reading this
//      rank's rows when the next step's normalisation rewrites them.
//
// Bytes over NVLink per rank: (world-1)/world of the rows (reduce) plus
// (world-1)/world of agg (broadcast), against 2(world-1)/world of the rows for
// a ring all-reduce.  Flags are per-step epochs (monotonic, never reset, wrap
// safe), so no clearing pass is needed.  Every wait is bounded (2 s of
// %globaltimer); on expiry the kernel raises KVC_DEV_TIMEOUT in the error flag
// and completes.  The grid never exceeds one wave of resident CTAs.
//
// Flag words of one rank: ready[world], pushed[world], CTA counter, started
// epoch, then four uint64 %globaltimer stamps of the last step on this rank:
// first CTA start, first CTA to see every rank ready, last CTA done, every
// rank's "agg pushed" seen (rank skew = stamp1 - stamp0, exchange = stamp3 - stamp1).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "kvc_common.cuh"

namespace kvc {

constexpr uint64_t kTpWaitNs = 2000000000ull;
constexpr int kTpThreads = 256;
constexpr int kTpMaxLayers = 512;

struct TpArgs {
  const float* const* rows;  // [world] each rank's rows[L][tok_total]
  float* const* agg;         // [world] each rank's agg[tok_total]
  int32_t* const* flags;     // [world] each rank's flag words
  const int32_t* tokens;
  const int32_t* page_off;
  int32_t* error_flag;
  int64_t tok_total;
  int world, rank, L, R, layer_agg;
  int32_t epoch;
};

__host__ __device__ constexpr int tp_stamp_word(int world) { return 2 * world + 2; }

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

// Valid tokens (0..4) of the quad starting at token `tok` of the page-padded space.
__device__ __forceinline__ int quad_valid(const TpArgs& a, int64_t tok) {
  const int r = request_of_page(a.page_off, a.R, (int)(tok >> 7));
  const int t = (int)(tok - (int64_t)__ldg(a.page_off + r) * kBlock);
  return max(0, min(4, __ldg(a.tokens + r) - t));
}

// W: the world size when it is compiled in (1, 2, 4, 8), else 0 (runtime, loads in groups of 8).
template <int W>
__global__ void __launch_bounds__(kTpThreads) tp_reduce_push_kernel(const __grid_constant__ TpArgs a) {
  extern __shared__ float4 tp_sm[];  // [L][Q] per-layer maxima, then [Q] finished quads
  __shared__ int ok;
  __shared__ const float* rows_s[KVC_TP_MAX_WORLD];
  __shared__ float* agg_s[KVC_TP_MAX_WORLD];
  const int world = W ? W : a.world;
  for (int p = threadIdx.x; p < world; p += blockDim.x) {
    rows_s[p] = a.rows[p];
    agg_s[p] = a.agg[p];
  }
  int32_t* mine = a.flags[a.rank];
  unsigned long long* stamps = reinterpret_cast<unsigned long long*>(mine + tp_stamp_word(world));
  if (threadIdx.x == 0) {
    if (atomicExch(mine + 2 * world + 1, a.epoch) != a.epoch) {  // the first CTA of this step announces
      stamps[1] = ~0ull;
      stamps[0] = tp_now_ns();
      __threadfence_system();  // this rank's rows (previous kernel) and the stamps before "rows ready"
      for (int p = 0; p < world; ++p) st_release_sys(a.flags[p] + a.rank, a.epoch);
    }
    ok = wait_epochs(mine, world, a.epoch);
    if (ok) atomicMin(stamps + 1, (unsigned long long)tp_now_ns());
    else raise_flag(a.error_flag, KVC_DEV_TIMEOUT);
  }
  __syncthreads();
  const int LT = min(a.L, 64);            // layer threads per quad
  const int Q = kTpThreads / LT;          // quads per group
  float4* part = tp_sm;                   // [L][Q]
  float4* done = tp_sm + (int64_t)a.L * Q;  // [Q]
  if (ok) {
    const int64_t quads = a.tok_total >> 2;
    const int64_t per = (quads + world - 1) / world;
    const int64_t lo = (int64_t)a.rank * per;
    const int64_t hi = min64(lo + per, quads);
    const int qi = threadIdx.x / LT, lt = threadIdx.x % LT;
    for (int64_t g0 = lo + (int64_t)blockIdx.x * Q; g0 < hi; g0 += (int64_t)gridDim.x * Q) {
      const int64_t q = g0 + qi;
      if (qi < Q && q < hi && quad_valid(a, q << 2) > 0) {
        for (int l = lt; l < a.L; l += LT) {
          const int64_t i = (int64_t)l * a.tok_total + (q << 2);
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
          part[l * Q + qi] = m;
        }
      }
      __syncthreads();
      if (threadIdx.x < Q && g0 + threadIdx.x < hi) {
        const int64_t tok = (g0 + threadIdx.x) << 2;
        const int nv = quad_valid(a, tok);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);  // page padding, as kvc_aggregate_rows
        if (nv > 0) {
          float4 acc = part[threadIdx.x];
          for (int l = 1; l < a.L; ++l) {
            const float4 m = part[l * Q + threadIdx.x];
            acc = a.layer_agg == KVC_AGG_MEAN ? make_float4(acc.x + m.x, acc.y + m.y, acc.z + m.z, acc.w + m.w)
                                              : nan_max4(acc, m);
          }
          if (a.layer_agg == KVC_AGG_MEAN) {
            const float d = (float)a.L;
            acc = make_float4(__fdiv_rn(acc.x, d), __fdiv_rn(acc.y, d), __fdiv_rn(acc.z, d), __fdiv_rn(acc.w, d));
          }
          v = make_float4(nv > 0 ? finalize_score(acc.x) : 0.f, nv > 1 ? finalize_score(acc.y) : 0.f,
                          nv > 2 ? finalize_score(acc.z) : 0.f, nv > 3 ? finalize_score(acc.w) : 0.f);
        }
        done[threadIdx.x] = v;
      }
      __syncthreads();
      const int nq = (int)min64(Q, hi - g0);
      for (int k = threadIdx.x; k < nq * world; k += blockDim.x) {  // consecutive threads, consecutive quads
        const int qq = k % nq, p = k / nq;
        *reinterpret_cast<float4*>(agg_s[p] + ((g0 + qq) << 2)) = done[qq];
      }
      __syncthreads();  // part / done are rewritten by the next group
    }
  }
  __threadfence_system();  // this thread's peer stores before the completion count
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t* counter = mine + 2 * world;
    if (atomicAdd(counter, 1) == (int)gridDim.x - 1) {
      atomicExch(counter, 0);
      stamps[2] = tp_now_ns();
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(a.flags[p] + world + a.rank, a.epoch);
      if (!wait_epochs(mine + world, world, a.epoch)) raise_flag(a.error_flag, KVC_DEV_TIMEOUT);
      stamps[3] = tp_now_ns();
    }
  }
}

template <int W>
int tp_blocks_per_sm(size_t smem) {
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, tp_reduce_push_kernel<W>, kTpThreads, smem) != cudaSuccess ||
      b < 1) {
    cudaGetLastError();
    b = 1;
  }
  return b;
}

template <int W>
int launch_tp(const TpArgs& a, cudaStream_t st) {
  const int LT = std::min(a.L, 64), Q = kTpThreads / LT;
  const size_t smem = ((size_t)a.L * Q + Q) * sizeof(float4);
  const int64_t quads = a.tok_total / 4;
  const int64_t groups = ((quads + a.world - 1) / a.world + Q - 1) / Q;
  // one wave at most: every CTA is resident, so the first CTA's signal and
  // every CTA's wait run together
  const int64_t cap = (int64_t)sm_count() * tp_blocks_per_sm<W>(smem);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(groups, cap));
  tp_reduce_push_kernel<W><<<grid, kTpThreads, smem, st>>>(a);
  return launch_status();
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

extern "C" int kvc_tp_exchange_flag_words(int world) { return world > 0 ? tp_stamp_word(world) + 8 : 0; }

extern "C" int kvc_tp_exchange_stamp_word(int world) { return world > 0 ? tp_stamp_word(world) : 0; }

extern "C" int kvc_tp_exchange_max(const float* const* peer_rows, float* const* peer_agg, int32_t* const* peer_flags,
                                   int world, int rank, int num_layers, int total_pages, const int32_t* tokens,
                                   const int32_t* page_off, int num_requests, int layer_aggregation, int32_t epoch,
                                   int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(peer_rows && peer_agg && peer_flags && tokens && page_off, KVC_ENULL);
  KVC_CHECK_ARG(world >= 1 && world <= KVC_TP_MAX_WORLD && rank >= 0 && rank < world, KVC_EINVAL);
  KVC_CHECK_ARG(num_layers > 0 && total_pages >= 0 && num_requests >= 0 && epoch > 0, KVC_EINVAL);
  KVC_CHECK_ARG(num_layers <= kTpMaxLayers, KVC_EUNSUPPORTED);
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
  // every rank runs the kernel every step, even with no tokens, so the epochs
  // of all ranks advance together
  cudaStream_t st = (cudaStream_t)stream;
  switch (world) {
    case 1: return launch_tp<1>(a, st);
    case 2: return launch_tp<2>(a, st);
    case 4: return launch_tp<4>(a, st);
    case 8: return launch_tp<8>(a, st);
    default: return launch_tp<0>(a, st);
  }
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

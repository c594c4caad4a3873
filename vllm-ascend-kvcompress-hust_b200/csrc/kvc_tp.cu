// Tensor-parallel score sync over NVLink peer memory (sm_100a).
//
// Every TP rank scores its own KV heads.  The step's tokens are split into
// world equal ranges of 4-token quads; rank o "owns" range o and keeps an
// inbox [world source ranks][L layers][per quads][4] fp32 that every other
// rank has mapped through CUDA IPC.  Two kernels per rank replace the MAX
// all-reduce of the per-layer rows and the layer reduction after it:
//
//   push (kvc_tp_push_rows): normalisation and head max of this rank's heads
//     (the same arithmetic as kvc_normalize_aggregate, kvc_norm.cuh), each
//     quad's value stored straight into its owner's inbox -- plain peer
//     stores, so the NVLink traffic is writes issued while the kernel still
//     streams raw scores from HBM.  The last CTA signals "delivered" to every
//     rank.
//   exchange (kvc_tp_exchange_max): every CTA waits for every rank's
//     "delivered"; for its owned quads a CTA takes a group of Q quads with up
//     to 64 threads per quad, one per layer, each loading the world sources of
//     one (quad, layer) from the LOCAL inbox and keeping their NaN-propagating
//     max in shared memory; one thread per quad reduces the layers in order
//     (sequential fp32 sum / L, or max) and finalises exactly as
//     kvc_aggregate_rows does; consecutive threads store consecutive finished
//     quads into every rank's agg buffer.  The last CTA signals "agg pushed" to
//     every rank and waits for every rank's "agg pushed" before the kernel
//     ends, so the selection launched next reads complete scores, and no rank
//     still reads its inbox when the next step's pushes arrive.
//
// Bytes over NVLink per rank: (world-1)/world of its rows and (world-1)/world
// of the finished scores, all as stores.  Flags are per-step epochs
// (monotonic, never reset, wrap safe), so no clearing pass is needed.  Every
// wait is bounded (2 s of %globaltimer); on expiry the kernel raises
// KVC_DEV_TIMEOUT in the error flag and completes.  The exchange grid never
// exceeds one wave of resident CTAs.
//
// Flag words of one rank: delivered[world], pushed[world], exchange CTA
// counter, started epoch, push CTA counter, one spare, then four uint64
// %globaltimer stamps of the last exchange on this rank: first CTA start,
// first CTA to see every rank's rows delivered, last CTA done, every rank's
// "agg pushed" seen (rank skew = stamp1 - stamp0, exchange = stamp3 - stamp1).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "kvc_norm.cuh"

namespace kvc {

constexpr uint64_t kTpWaitNs = 2000000000ull;
constexpr int kTpThreads = 256;
constexpr int kTpMaxLayers = 512;

__host__ __device__ constexpr int tp_exch_counter(int world) { return 2 * world; }
__host__ __device__ constexpr int tp_started(int world) { return 2 * world + 1; }
__host__ __device__ constexpr int tp_push_counter(int world) { return 2 * world + 2; }
__host__ __device__ constexpr int tp_stamp_word(int world) { return 2 * world + 4; }

// Quads of the padded token space owned by each rank.
__host__ __device__ inline int64_t tp_quads_per_rank(int64_t tok_total, int world) {
  return (tok_total / 4 + world - 1) / world;
}

struct TpArgs {
  float* const* inbox;       // [world] each rank's inbox [world][L][per][4]
  float* const* agg;         // [world] each rank's agg[tok_total]
  int32_t* const* flags;     // [world] each rank's flag words
  const int32_t* tokens;
  const int32_t* page_off;
  int32_t* error_flag;
  int64_t tok_total;
  int64_t per;               // quads per owner
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

// Valid tokens (0..4) of the quad starting at token `tok` of the page-padded space.
__device__ __forceinline__ int quad_valid(const int32_t* page_off, const int32_t* tokens, int R, int64_t tok) {
  const int r = request_of_page(page_off, R, (int)(tok >> 7));
  const int t = (int)(tok - (int64_t)__ldg(page_off + r) * kBlock);
  return max(0, min(4, __ldg(tokens + r) - t));
}

// ---- push: normalise this rank's heads and deliver each quad to its owner ----

struct PushArgs {
  const float* raw;
  const float* mean;
  const float* den;
  const int32_t* tokens;
  const int32_t* page_off;
  float* const* inbox;
  int32_t* const* flags;
  int64_t per;
  int L, heads, total_pages, R, world, rank;
  int32_t epoch;
};

// QPT quads per thread per page group (8 * QPT pages): with few local heads
// the per-group staging (request lookup, head statistics) and the per-quad
// store dominate, so each thread takes several quads to amortise them and
// keep more loads in flight.  The arithmetic per quad is norm_quad's.
template <int QPT>
__global__ void __launch_bounds__(256) tp_push_rows_kernel(const __grid_constant__ PushArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  constexpr int NP = 8 * QPT;
  extern __shared__ float st[];  // [3][NP][heads]
  __shared__ NormPagesN<NP> np;
  __shared__ float* inbox_s[KVC_TP_MAX_WORLD];
  for (int p = threadIdx.x; p < a.world; p += blockDim.x) inbox_s[p] = a.inbox[p];
  const int l = blockIdx.y;
  // grid-stride over page groups: few CTAs, so one system fence per CTA
  for (int page0 = blockIdx.x * NP; page0 < a.total_pages; page0 += gridDim.x * NP) {
    norm_stage_n<NP>(np, st, page0, l, a.heads, a.total_pages, a.R, a.tokens, a.page_off, a.mean, a.den);
#pragma unroll
    for (int i = 0; i < QPT; ++i) {
      int64_t tok;
      float4 z;
      if (norm_quad_split<NP, 1>(np, st, a.raw, l, a.heads, a.total_pages, page0, threadIdx.x + 256 * i, 0, tok,
                                 z) > 0) {
        const int64_t q = tok >> 2;
        const int o = (int)(q / a.per);
        float* dst = inbox_s[o] + (((int64_t)a.rank * a.L + l) * a.per + (q - (int64_t)o * a.per)) * 4;
        *reinterpret_cast<float4*>(dst) = z;  // a peer store unless this rank owns the quad
      }
    }
    __syncthreads();  // np / st are restaged for the next group
  }
  // the CTA barrier orders every thread's stores before thread 0's system fence,
  // which is cumulative over them (release pattern), then the completion count
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    int32_t* counter = a.flags[a.rank] + tp_push_counter(a.world);
    if (atomicAdd(counter, 1) == (int)(gridDim.x * gridDim.y) - 1) {
      atomicExch(counter, 0);
      __threadfence_system();
      for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + a.rank, a.epoch);
    }
  }
}

// ---- exchange: reduce the owned quads from the local inbox, push the scores ----

// W: the world size when it is compiled in (1, 2, 4, 8), else 0 (runtime).
template <int W>
__global__ void __launch_bounds__(kTpThreads) tp_reduce_push_kernel(const __grid_constant__ TpArgs a) {
  // launched in plain stream order and without early dependents: its CTAs spin on
  // peer flags, so nothing else is let onto the SMs beside them
  extern __shared__ float4 tp_sm[];  // [L][Q] per-layer maxima, then [Q] finished quads
  __shared__ int ok;
  __shared__ float* agg_s[KVC_TP_MAX_WORLD];
  const int world = W ? W : a.world;
  for (int p = threadIdx.x; p < world; p += blockDim.x) agg_s[p] = a.agg[p];
  int32_t* mine = a.flags[a.rank];
  unsigned long long* stamps = reinterpret_cast<unsigned long long*>(mine + tp_stamp_word(world));
  if (threadIdx.x == 0) {
    if (atomicExch(mine + tp_started(world), a.epoch) != a.epoch) {  // the first CTA of this step
      stamps[1] = ~0ull;
      stamps[0] = tp_now_ns();
    }
    ok = wait_epochs(mine, world, a.epoch);  // every rank's rows delivered to this inbox
    if (ok) atomicMin(stamps + 1, (unsigned long long)tp_now_ns());
    else raise_flag(a.error_flag, KVC_DEV_TIMEOUT);
  }
  __syncthreads();
  const int LT = min(a.L, 64);            // layer threads per quad
  const int Q = kTpThreads / LT;          // quads per group
  float4* part = tp_sm;                   // [L][Q]
  float4* done = tp_sm + (int64_t)a.L * Q;  // [Q]
  if (ok) {
    const float4* inbox = reinterpret_cast<const float4*>(a.inbox[a.rank]);
    const int64_t quads = a.tok_total >> 2;
    const int64_t lo = (int64_t)a.rank * a.per;
    const int64_t hi = min64(lo + a.per, quads);
    const int64_t src_stride = (int64_t)a.L * a.per;  // float4s between two sources' blocks
    const int qi = threadIdx.x / LT, lt = threadIdx.x % LT;
    for (int64_t g0 = lo + (int64_t)blockIdx.x * Q; g0 < hi; g0 += (int64_t)gridDim.x * Q) {
      const int64_t q = g0 + qi;
      if (qi < Q && q < hi && quad_valid(a.page_off, a.tokens, a.R, q << 2) > 0) {
        for (int l = lt; l < a.L; l += LT) {
          const float4* src = inbox + (int64_t)l * a.per + (q - lo);
          float4 m = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
          if constexpr (W > 0) {
            float4 x[W];
#pragma unroll
            for (int p = 0; p < W; ++p) x[p] = src[p * src_stride];
#pragma unroll
            for (int p = 0; p < W; ++p) m = nan_max4(m, x[p]);
          } else {
            for (int p0 = 0; p0 < world; p0 += 8) {
              float4 x[8];
#pragma unroll
              for (int k = 0; k < 8; ++k)
                if (p0 + k < world) x[k] = src[(p0 + k) * src_stride];
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
        const int nv = quad_valid(a.page_off, a.tokens, a.R, tok);
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
          v = make_float4(finalize_score(acc.x), nv > 1 ? finalize_score(acc.y) : 0.f,
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
  // the CTA barrier orders every thread's peer stores before thread 0's
  // system fence, which is cumulative over them, then the completion count
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    int32_t* counter = mine + tp_exch_counter(world);
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
  const int64_t groups = (a.per + Q - 1) / Q;
  // one wave at most: every CTA is resident, so every CTA's wait runs together
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

extern "C" int64_t kvc_tp_exchange_inbox_floats(int world, int num_layers, int total_pages) {
  if (world < 1 || num_layers < 1 || total_pages < 0) return 0;
  return (int64_t)world * num_layers * tp_quads_per_rank((int64_t)total_pages * kBlock, world) * 4;
}

extern "C" int kvc_tp_push_rows(const float* raw, int num_layers, int heads, int total_pages, const float* mean,
                                const float* denom, const int32_t* tokens, const int32_t* page_off, int num_requests,
                                float* const* peer_inbox, int32_t* const* peer_flags, int world, int rank,
                                int32_t epoch, void* stream) {
  KVC_CHECK_ARG(raw && mean && denom && tokens && page_off && peer_inbox && peer_flags, KVC_ENULL);
  KVC_CHECK_ARG(world >= 1 && world <= KVC_TP_MAX_WORLD && rank >= 0 && rank < world, KVC_EINVAL);
  KVC_CHECK_ARG(num_layers > 0 && num_layers <= 65535 && heads > 0 && total_pages >= 0 && num_requests >= 0 &&
                    epoch > 0,
                KVC_EINVAL);
  KVC_CHECK_ARG(aligned(raw, 16), KVC_EALIGN);
  const int qpt = heads <= 8 ? 4 : heads <= 16 ? 2 : 1;  // quads per thread per page group
  const int np = 8 * qpt;
  const size_t smem = (size_t)3 * np * heads * sizeof(float);
  KVC_CHECK_ARG(smem <= 48 * 1024, KVC_EUNSUPPORTED);
  PushArgs a{};
  a.raw = raw;
  a.mean = mean;
  a.den = denom;
  a.tokens = tokens;
  a.page_off = page_off;
  a.inbox = peer_inbox;
  a.flags = peer_flags;
  a.per = tp_quads_per_rank((int64_t)total_pages * kBlock, world);
  a.L = num_layers;
  a.heads = heads;
  a.total_pages = total_pages;
  a.R = num_requests;
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  // every rank launches every step, even with no tokens, so the epochs of all ranks advance together;
  // up to eight CTAs per SM (the thread limit) over all layers, each striding
  // over page groups: each group is a chain of dependent loads (request
  // lookup, head statistics, raw scores), so many CTAs in flight hide it
  const int groups = std::max(1, (total_pages + np - 1) / np);
  const int per_layer = std::max(1, std::min(groups, (8 * sm_count() + num_layers - 1) / num_layers));
  const dim3 grid((unsigned)per_layer, (unsigned)num_layers);
  cudaStream_t st = (cudaStream_t)stream;
  if (qpt == 4) launch_dep(tp_push_rows_kernel<4>, grid, dim3(256), smem, st, a);
  else if (qpt == 2) launch_dep(tp_push_rows_kernel<2>, grid, dim3(256), smem, st, a);
  else launch_dep(tp_push_rows_kernel<1>, grid, dim3(256), smem, st, a);
  return launch_status();
}

extern "C" int kvc_tp_exchange_max(float* const* peer_inbox, float* const* peer_agg, int32_t* const* peer_flags,
                                   int world, int rank, int num_layers, int total_pages, const int32_t* tokens,
                                   const int32_t* page_off, int num_requests, int layer_aggregation, int32_t epoch,
                                   int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(peer_inbox && peer_agg && peer_flags && tokens && page_off, KVC_ENULL);
  KVC_CHECK_ARG(world >= 1 && world <= KVC_TP_MAX_WORLD && rank >= 0 && rank < world, KVC_EINVAL);
  KVC_CHECK_ARG(num_layers > 0 && total_pages >= 0 && num_requests >= 0 && epoch > 0, KVC_EINVAL);
  KVC_CHECK_ARG(num_layers <= kTpMaxLayers, KVC_EUNSUPPORTED);
  KVC_CHECK_ARG(layer_aggregation == KVC_AGG_MEAN || layer_aggregation == KVC_AGG_MAX, KVC_EINVAL);
  TpArgs a{};
  a.inbox = peer_inbox;
  a.agg = peer_agg;
  a.flags = peer_flags;
  a.tokens = tokens;
  a.page_off = page_off;
  a.error_flag = error_flag;
  a.tok_total = (int64_t)total_pages * kBlock;
  a.per = tp_quads_per_rank(a.tok_total, world);
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

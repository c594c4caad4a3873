// Ragged, segmented top-budget selection (global and V3 policies) on sm_100a.
//
// One CTA per (segment, request).  The V3 integer plan is evaluated in closed
// form per segment, so CTAs never communicate:
//   M = T - prefix - recent, E = T - budget
//   segment s = [P0 + M*s/S, P0 + M*(s+1)/S), evictions E*(stop-P0)/M - E*(start-P0)/M
//   output offset of s = prefix + (start - P0) - E*(start-P0)/M  (telescoping sum)
// The global policy is the one-segment case (protected tokens outrank every
// finite middle score, so "protected + top of the middle" equals top-budget
// with protected scores set to +inf).
//
// Within a segment the k-th largest score is found by a 4-pass MSB-first radix
// select over order-preserving 32-bit keys (8-bit digits, shared-memory
// histograms), then one ordered pass writes the kept positions ascending:
// keys above the threshold, plus the first (lowest-position) keys equal to it.
#include "kvc_common.cuh"

namespace kvc {

constexpr int kSelThreads = 512;
constexpr int kSelWarps = kSelThreads / 32;

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive scan of one 32-bit value; returns the block total too.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_tot, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kSelWarps ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kSelWarps) warp_tot[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  const uint32_t before = (warp ? warp_tot[warp - 1] : 0u) + x - v;
  total = warp_tot[kSelWarps - 1];
  __syncthreads();
  return before;
}

struct SelectArgs {
  const float* agg;
  const int32_t* tokens;
  const int32_t* page_off;
  int64_t* keep;
  int32_t* error_flag;
  int R, budget, prefix, recent, segments, policy;
};

__global__ void __launch_bounds__(kSelThreads) select_kernel(const __grid_constant__ SelectArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_tot[kSelWarps];
  __shared__ uint32_t s_digit, s_above;
  const int s = blockIdx.x, r = blockIdx.y;
  const int S = a.policy == KVC_POLICY_GLOBAL ? 1 : a.segments;
  if (s >= S) return;
  const int64_t T = a.tokens[r];
  const int64_t B = a.budget;
  const int64_t prefix = min64(a.prefix, T);
  const int64_t recent = min64(a.recent, T - prefix);
  const int64_t M = T - prefix - recent;
  const int64_t E = T - B;
  if (B > T || B <= 0 || prefix + recent > B || E > M || E < 0) {
    if (threadIdx.x == 0 && s == 0) raise_flag(a.error_flag, KVC_DEV_BUDGET);
    return;
  }
  const float* sc = a.agg + (int64_t)a.page_off[r] * kBlock;
  int64_t* out = a.keep + (int64_t)r * B;
  if (s == 0) {
    for (int64_t i = threadIdx.x; i < prefix; i += blockDim.x) out[i] = i;
    for (int64_t i = threadIdx.x; i < recent; i += blockDim.x) out[B - recent + i] = T - recent + i;
  }
  if (M <= 0) return;
  const int64_t start = prefix + M * s / S;
  const int64_t stop = prefix + M * (s + 1) / S;
  const int64_t n = stop - start;
  const int64_t ev_before = E * (start - prefix) / M;
  const int64_t ev_after = E * (stop - prefix) / M;
  const int64_t k = n - (ev_after - ev_before);
  const int64_t base = prefix + (start - prefix) - ev_before;
  if (n <= 0 || k <= 0) return;
  if (k == n) {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[base + i] = start + i;
    return;
  }
  const float* seg = sc + start;

  // ---- radix select of the k-th largest key ------------------------------
  uint32_t want = 0, mask = 0;
  uint32_t krem = (uint32_t)k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t key = order_key(__ldg(seg + i));
      if ((key & mask) == want) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane L owns digits 255-8L .. 248-8L (descending); find the digit where
      // the count of keys with a larger digit first reaches krem
      const int lane = threadIdx.x;
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - 8 * lane - j];
        sum += c[j];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      uint32_t above = incl - sum;  // keys in higher digits than this lane's range
      if (above < krem && krem <= incl) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (above < krem && krem <= above + c[j]) {
            s_digit = 255 - 8 * lane - j;
            s_above = above;
          }
          above += c[j];
        }
      }
    }
    __syncthreads();
    want |= s_digit << shift;
    mask |= 255u << shift;
    krem -= s_above;
    __syncthreads();
  }
  const uint32_t thr = want;   // key of the k-th largest score
  const uint32_t keq = krem;   // keys equal to thr that are kept (lowest positions)

  // ---- ordered write of kept positions ------------------------------------
  uint32_t run_gt = 0, run_eq = 0;
  for (int64_t c0 = 0; c0 < n; c0 += blockDim.x) {
    const int64_t i = c0 + threadIdx.x;
    uint32_t gt = 0, eq = 0;
    if (i < n) {
      const uint32_t key = order_key(__ldg(seg + i));
      gt = key > thr;
      eq = key == thr;
    }
    uint32_t tot;
    const uint32_t ex = block_exclusive_scan((eq << 16) | gt, warp_tot, tot);
    const uint32_t eq_before = run_eq + (ex >> 16);
    const uint32_t gt_before = run_gt + (ex & 0xffffu);
    if (gt || (eq && eq_before < keq)) out[base + gt_before + min(eq_before, keq)] = start + i;
    run_gt += tot & 0xffffu;
    run_eq += tot >> 16;
  }
}

}  // namespace kvc

using namespace kvc;

extern "C" int kvc_select_keep(const float* agg, const int32_t* tokens, const int32_t* page_off, int R,
                               int budget, int prefix, int recent, int segments, int policy,
                               int64_t* keep_out, int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(agg && tokens && page_off && keep_out, KVC_ENULL);
  KVC_CHECK_ARG(R >= 0 && R <= 65535 && budget > 0 && prefix >= 0 && recent >= 0 && prefix + recent <= budget,
                KVC_EINVAL);
  KVC_CHECK_ARG(policy == KVC_POLICY_GLOBAL || (policy == KVC_POLICY_V3 && segments > 0 && segments <= 65535),
                KVC_EINVAL);
  if (R == 0) return KVC_OK;
  SelectArgs a{agg, tokens, page_off, keep_out, error_flag, R, budget, prefix, recent, segments, policy};
  const int S = policy == KVC_POLICY_GLOBAL ? 1 : segments;
  launch_dep(select_kernel, dim3(S, R), dim3(kSelThreads), 0, (cudaStream_t)stream, a);
  return launch_status();
}

// Per-(token, layer) normalisation and head max, shared by the row writer
// (kvc_normalize_aggregate) and the tensor-parallel push (kvc_tp_push_rows), so
// both produce bit-identical values.
//
// A CTA of 256 threads covers NP pages of one scoring layer; each token quad
// (4 consecutive tokens) is handled by HS lanes that split its query heads, or
// (HS = 1) one lane may take several quads.  A lane loads each of its heads'
// raw scores of the 4 tokens as one 16-byte vector (page-major raw: a page's
// 128 scores of one head are contiguous).  The request of each page and its
// per-head mean, denominator and reciprocal for the layer are staged in shared
// memory first (norm_stage_n).
#pragma once

#include "kvc_common.cuh"

namespace kvc {

// a / b from the correctly rounded reciprocal rcp = RN(1/b): q0 = RN(a * rcp),
// residual r = a - q0 * b (exact by FMA), q = RN(q0 + r * rcp).  Markstein's
// correction step (P. Markstein, "Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990) returns the
// correctly rounded quotient for normal operands, as IEEE division would; the
// denominators here are >= 1e-3 and the numerators finite or NaN/inf, which
// propagate the same way.  Falls back to the division when a, b are not finite.
__device__ __forceinline__ float div_by(float a, float b, float rcp) {
  if (!isfinite(a) || !isfinite(b)) return __fdiv_rn(a, b);
  const float q0 = __fmul_rn(a, rcp);
  const float r = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(r, rcp, q0);
}

template <int NP>
struct NormPagesN {
  int req[NP];
  int64_t start[NP];  // first token of the page's request in the padded space
  int ntok[NP];
};

// Stage the CTA's page table and layer l's statistics ([NP][heads] mean, den,
// 1/den in `st`).  Every thread of the CTA calls it; it ends synchronised.
template <int NP>
__device__ __forceinline__ void norm_stage_n(NormPagesN<NP>& np, float* st, int page0, int l, int heads,
                                             int total_pages, int R, const int32_t* __restrict__ tokens,
                                             const int32_t* __restrict__ page_off, const float* __restrict__ mean,
                                             const float* __restrict__ den) {
  if (threadIdx.x < NP) {
    const int p = page0 + threadIdx.x;
    int r = 0;
    if (p < total_pages) {
      r = request_of_page(page_off, R, p);
      np.start[threadIdx.x] = (int64_t)__ldg(page_off + r) * kBlock;
      np.ntok[threadIdx.x] = __ldg(tokens + r);
    }
    np.req[threadIdx.x] = r;
  }
  __syncthreads();
  float* mu_s = st;
  float* dn_s = st + NP * heads;
  float* rc_s = st + 2 * NP * heads;
  for (int i = threadIdx.x; i < NP * heads; i += blockDim.x) {
    const int slot = i / heads;
    if (page0 + slot >= total_pages) continue;
    const int64_t g = ((int64_t)l * R + np.req[slot]) * heads + i % heads;
    mu_s[i] = __ldg(mean + g);
    const float d = __ldg(den + g);
    dn_s[i] = d;
    rc_s[i] = __frcp_rn(d);
  }
  __syncthreads();
}

// The head max of (raw - mean) / den for the 4 tokens of quad `quad` of the
// CTA's pages (its token index in the padded space in `tok`; 0 for page
// padding), with the heads shared by HS adjacent lanes: the thread of
// (quad, slice) covers heads slice, slice + HS, ..., and the HS lanes of a
// quad combine their maxima by shuffles (every lane of the warp must call it
// when HS > 1).
// Pages of NP per CTA, 32 quads of 4 tokens per page.  Returns the valid
// token count of the quad; z is complete in every lane of the quad.
template <int NP, int HS>
__device__ __forceinline__ int norm_quad_split(const NormPagesN<NP>& np, const float* st,
                                               const float* __restrict__ raw, int l, int heads, int total_pages,
                                               int page0, int quad, int slice, int64_t& tok, float4& z) {
  const int slot = quad >> 5;
  const int p = page0 + slot;
  tok = (int64_t)p * kBlock + (quad & 31) * 4;
  float4 m4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  int t = 0, n = 0;
  if (p < total_pages) {
    t = (int)(tok - np.start[slot]);
    n = np.ntok[slot];
    const float* mu = st + slot * heads;
    const float* dn = st + NP * heads + slot * heads;
    const float* rc = st + 2 * NP * heads + slot * heads;
    const float4* rl = reinterpret_cast<const float4*>(raw + ((int64_t)l * total_pages + p) * heads * kBlock +
                                                       (tok & (kBlock - 1)));
    if (t < n) {
      constexpr int U = HS == 1 ? 4 : 2;  // heads of this slice whose loads are in flight together
      for (int h0 = slice; h0 < heads; h0 += U * HS) {
        float4 x[U];
#pragma unroll
        for (int k = 0; k < U; ++k)
          if (h0 + k * HS < heads) x[k] = __ldg(rl + (int64_t)(h0 + k * HS) * (kBlock / 4));
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int h = h0 + k * HS;
          if (h < heads) {
            const float m = mu[h], d = dn[h], c = rc[h];
            m4.x = nan_max(m4.x, div_by(x[k].x - m, d, c));
            m4.y = nan_max(m4.y, div_by(x[k].y - m, d, c));
            m4.z = nan_max(m4.z, div_by(x[k].z - m, d, c));
            m4.w = nan_max(m4.w, div_by(x[k].w - m, d, c));
          }
        }
      }
    }
  }
#pragma unroll
  for (int o = 1; o < HS; o <<= 1) {
    m4.x = nan_max(m4.x, __shfl_xor_sync(0xffffffffu, m4.x, o));
    m4.y = nan_max(m4.y, __shfl_xor_sync(0xffffffffu, m4.y, o));
    m4.z = nan_max(m4.z, __shfl_xor_sync(0xffffffffu, m4.z, o));
    m4.w = nan_max(m4.w, __shfl_xor_sync(0xffffffffu, m4.w, o));
  }
  z = make_float4(t + 0 < n ? m4.x : 0.f, t + 1 < n ? m4.y : 0.f, t + 2 < n ? m4.z : 0.f, t + 3 < n ? m4.w : 0.f);
  return t < n ? min(4, n - t) : 0;
}

}  // namespace kvc

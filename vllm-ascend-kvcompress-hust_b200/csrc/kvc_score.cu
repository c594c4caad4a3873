// Trigonometric key scoring for TriAttention on sm_100a.
//
// Pipeline (all launches on the caller's stream):
//   prepare_coef   : per (request, scoring layer) phase means and the folded
//                    per (kv head, q head, frequency) coefficients a, b, e
//   score_mean     : streams every 128-token page of K once per scoring layer,
//                    raw[l][h*G+g][token] = sum_f kr*a + ki*b + |k|*e (+ q_pass.k)
//                    and per-page moments (sum, M2) of every query head
//   head_stats     : fp64 Chan combination of the page moments -> mean, var
//   normalize      : z = (raw - mean) / sqrt(max(var, 1e-6)), max over heads,
//                    layer mean/max (or per-layer rows for the TP all-reduce)
//   aggregate_rows : layer reduction after the TP all-reduce
//
// Algebra: the reference scores  sum_f s*((qr*kr + qi*ki)*c - (qi*kr - qr*ki)*sn)
// which equals  sum_f kr*(s*(qr*c - qi*sn)) + ki*(s*(qi*c + qr*sn)); folding the
// per-request phase (c, sn) into a and b once per (request, layer) leaves three
// FMAs per (token, q head, frequency) in the streaming loop.
#include "kvc_common.cuh"
#include "kvc_norm.cuh"

namespace kvc {

__host__ __device__ constexpr int coef_group_stride(int g) { return (3 * g + 3) & ~3; }

// --------------------------------------------------------------------------
// coefficient preparation
// --------------------------------------------------------------------------

struct PrepArgs {
  const float* omega;      // [L][F]
  const float* offsets;    // [n_off]
  const int64_t* round_start;  // [R]
  const float* q_real;     // [L][kvh][G][F]
  const float* q_imag;
  const float* scale;
  const float* extra;
  float* coef;
  int n_off, R, L, kvh, G, F, aggregation;
  int64_t block_floats;    // floats per (r, l, h)
};

__global__ void __launch_bounds__(256) prepare_coef_kernel(PrepArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  extern __shared__ float sm[];
  float* cmean = sm;              // [F]
  float* smean = sm + a.F;        // [F]
  float* ctab = sm + 2 * a.F;     // [n_off][F]  (max aggregation only)
  float* stab = ctab + a.n_off * a.F;
  const int l = blockIdx.x, r = blockIdx.y;
  const float rs = (float)a.round_start[r];
  for (int f = threadIdx.x; f < a.F; f += blockDim.x) {
    const float w = a.omega[l * a.F + f];
    float cs = 0.f, ss = 0.f;
    for (int o = 0; o < a.n_off; ++o) {
      // fp32 (offset + round_start) then * omega, as the reference forms phases
      const float ph = __fmul_rn(__fadd_rn(a.offsets[o], rs), w);
      float s, c;
      sincosf(ph, &s, &c);
      cs += c;
      ss += s;
      if (a.aggregation == KVC_AGG_MAX) {
        ctab[o * a.F + f] = c;
        stab[o * a.F + f] = s;
      }
    }
    const float inv = 1.0f / (float)a.n_off;
    cmean[f] = cs * inv;
    smean[f] = ss * inv;
  }
  __syncthreads();
  const int CG = coef_group_stride(a.G);
  const int64_t total = (int64_t)a.kvh * a.G * a.F;
  for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
    const int f = i % a.F;
    const int g = (i / a.F) % a.G;
    const int h = i / ((int64_t)a.F * a.G);
    const int64_t src = ((int64_t)(l * a.kvh + h) * a.G + g) * a.F + f;
    const float qr = a.q_real[src], qi = a.q_imag[src], sc = a.scale[src], ex = a.extra[src];
    float* blk = a.coef + ((int64_t)(r * a.L + l) * a.kvh + h) * a.block_floats;
    const float c = cmean[f], s = smean[f];
    blk[f * CG + g] = sc * (qr * c - qi * s);
    blk[f * CG + a.G + g] = sc * (qi * c + qr * s);
    blk[f * CG + 2 * a.G + g] = ex * sc;
    if (g == 0)
      for (int pad = 3 * a.G; pad < CG; ++pad) blk[f * CG + pad] = 0.f;
    if (a.aggregation == KVC_AGG_MAX) {
      // per-offset coefficients [o][f][2G]: a_o, b_o
      float* tab = blk + (int64_t)a.F * CG;
      for (int o = 0; o < a.n_off; ++o) {
        const float co = ctab[o * a.F + f], so = stab[o * a.F + f];
        tab[((int64_t)o * a.F + f) * 2 * a.G + g] = sc * (qr * co - qi * so);
        tab[((int64_t)o * a.F + f) * 2 * a.G + a.G + g] = sc * (qi * co + qr * so);
      }
    }
  }
}

// --------------------------------------------------------------------------
// paged scorer (mean over future offsets)
// --------------------------------------------------------------------------

constexpr int kMaxLayers = 512;

struct ScoreArgs {
  const void* k_layers[kMaxLayers];
  int64_t block_stride;   // elements
  int64_t num_blocks;
  const int64_t* src_blocks;
  const int64_t* src_block_off;
  const int32_t* tokens;
  const int32_t* page_off;
  const float* coef;
  const float* q_pass_t;  // [L][kvh][P][G]
  float* raw;
  float* partial;
  int32_t* error_flag;
  int64_t coef_block;     // floats per (r, l, h)
  int64_t tok_total;
  int L, kvh, D, F, P, R, total_pages, n_off;
  int warp_floats;        // smem floats per warp
};

constexpr int kScoreWarps = 8;
constexpr int kTokPerLane = kBlock / 32;  // 4


// Coefficients of one frequency/dim from shared memory (broadcast reads).
template <int N>
__device__ __forceinline__ void load_coefs(const float* p, float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
      const float4 t = reinterpret_cast<const float4*>(p)[q];
      v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < N; ++q) v[q] = p[q];
  }
}

// One frequency of the rotary part for the lane's 4 tokens.
template <int G, class E, int J>
__device__ __forceinline__ void rope_freq(const float* cc, const uint4 (&kr)[kTokPerLane],
                                          const uint4 (&ki)[kTokPerLane], float (&acc)[kTokPerLane][G]) {
  constexpr int CG = coef_group_stride(G);
  float cv[CG];
  load_coefs<CG>(cc + J * CG, cv);
#pragma unroll
  for (int i = 0; i < kTokPerLane; ++i) {
    const float xr = elem8<J>(kr[i], E{});
    const float xi = elem8<J>(ki[i], E{});
    const float m = sqrtf(xr * xr + xi * xi);
#pragma unroll
    for (int g = 0; g < G; ++g)
      acc[i][g] = fmaf(m, cv[2 * G + g], fmaf(xi, cv[G + g], fmaf(xr, cv[g], acc[i][g])));
  }
}

template <int G, class E>
__device__ __forceinline__ void rope_chunk(const float* cc, const uint4 (&kr)[kTokPerLane],
                                           const uint4 (&ki)[kTokPerLane], float (&acc)[kTokPerLane][G]) {
  rope_freq<G, E, 0>(cc, kr, ki, acc);
  rope_freq<G, E, 1>(cc, kr, ki, acc);
  rope_freq<G, E, 2>(cc, kr, ki, acc);
  rope_freq<G, E, 3>(cc, kr, ki, acc);
  rope_freq<G, E, 4>(cc, kr, ki, acc);
  rope_freq<G, E, 5>(cc, kr, ki, acc);
  rope_freq<G, E, 6>(cc, kr, ki, acc);
  rope_freq<G, E, 7>(cc, kr, ki, acc);
}

// One unrotated dim: acc += k_pass * q_pass for every query head.
template <int G, class E, int J>
__device__ __forceinline__ void pass_dim(const float* qc, const uint4 (&kp)[kTokPerLane],
                                         float (&acc)[kTokPerLane][G]) {
  float q[G];
  load_coefs<G>(qc + J * G, q);
#pragma unroll
  for (int i = 0; i < kTokPerLane; ++i) {
    const float x = elem8<J>(kp[i], E{});
#pragma unroll
    for (int g = 0; g < G; ++g) acc[i][g] = fmaf(x, q[g], acc[i][g]);
  }
}

template <int G, class E>
__device__ __forceinline__ void pass_chunk(const float* qc, const uint4 (&kp)[kTokPerLane],
                                           float (&acc)[kTokPerLane][G]) {
  pass_dim<G, E, 0>(qc, kp, acc);
  pass_dim<G, E, 1>(qc, kp, acc);
  pass_dim<G, E, 2>(qc, kp, acc);
  pass_dim<G, E, 3>(qc, kp, acc);
  pass_dim<G, E, 4>(qc, kp, acc);
  pass_dim<G, E, 5>(qc, kp, acc);
  pass_dim<G, E, 6>(qc, kp, acc);
  pass_dim<G, E, 7>(qc, kp, acc);
}

// Page moments of one query head over the valid tokens of a page, then store.
template <int G>
__device__ __forceinline__ void page_epilogue(const ScoreArgs& a, float (&acc)[kTokPerLane][G],
                                              int lane, int valid, int l, int h, int p) {
  const int heads = a.kvh * G;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* row = a.raw + (((int64_t)l * a.total_pages + p) * heads + h * G + g) * kBlock;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kTokPerLane; ++i) {
      const int t = lane + 32 * i;
      if (t < valid) {
        row[t] = acc[i][g];
        s += acc[i][g];
      }
    }
    s = warp_sum(s);
    const float mu = s / (float)valid;
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < kTokPerLane; ++i) {
      const int t = lane + 32 * i;
      if (t < valid) {
        const float x = acc[i][g] - mu;
        d = fmaf(x, x, d);
      }
    }
    d = warp_sum(d);
    if (lane == 0) {
      float2* out = reinterpret_cast<float2*>(a.partial) + ((int64_t)l * a.total_pages + p) * heads + h * G + g;
      *out = make_float2(s, d);
    }
  }
}

// Locate the page of a work unit; returns false (and flags) when the block id is bad.
__device__ __forceinline__ bool unit_page(const ScoreArgs& a, int p, int& r, int& valid, int64_t& blk) {
  r = request_of_page(a.page_off, a.R, p);
  const int pl = p - __ldg(a.page_off + r);
  valid = min(kBlock, __ldg(a.tokens + r) - pl * kBlock);
  blk = __ldg(a.src_blocks + __ldg(a.src_block_off + r) + pl);
  if (valid <= 0) return false;
  if (blk < 0 || blk >= a.num_blocks) {
    raise_flag(a.error_flag, KVC_DEV_BLOCK_RANGE);
    return false;
  }
  return true;
}

template <int G, class E>
__global__ void __launch_bounds__(kScoreWarps * 32, 2) score_mean_kernel(const __grid_constant__ ScoreArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  extern __shared__ float4 smem4[];
  constexpr int CG = coef_group_stride(G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* cf = reinterpret_cast<float*>(smem4) + warp * a.warp_floats;
  float* qp = cf + a.F * CG;
  const int64_t units = (int64_t)a.L * a.total_pages * a.kvh;
  const int row = a.kvh * a.D;  // elements per token row
  for (int64_t u = (int64_t)blockIdx.x * kScoreWarps + warp; u < units;
       u += (int64_t)gridDim.x * kScoreWarps) {
    const int h = u % a.kvh;
    const int p = (u / a.kvh) % a.total_pages;
    const int l = u / ((int64_t)a.kvh * a.total_pages);
    int r, valid;
    int64_t blk;
    if (!unit_page(a, p, r, valid, blk)) continue;
    // stage this (request, layer, head)'s coefficients in the warp's slice
    {
      const float4* src = reinterpret_cast<const float4*>(a.coef + ((int64_t)(r * a.L + l) * a.kvh + h) * a.coef_block);
      float4* dst = reinterpret_cast<float4*>(cf);
      for (int i = lane; i < a.F * CG / 4; i += 32) dst[i] = __ldg(src + i);
      if (a.P) {
        const float4* ps = reinterpret_cast<const float4*>(a.q_pass_t + (int64_t)(l * a.kvh + h) * a.P * G);
        float4* pd = reinterpret_cast<float4*>(qp);
        for (int i = lane; i < a.P * G / 4; i += 32) pd[i] = __ldg(ps + i);
      }
    }
    __syncwarp();
    const uint16_t* base = reinterpret_cast<const uint16_t*>(a.k_layers[l]) + blk * a.block_stride + (int64_t)h * a.D;
    float acc[kTokPerLane][G];
#pragma unroll
    for (int i = 0; i < kTokPerLane; ++i)
#pragma unroll
      for (int g = 0; g < G; ++g) acc[i][g] = 0.f;

#pragma unroll 1
    for (int c = 0; c < a.F / 8; ++c) {
      uint4 kr[kTokPerLane], ki[kTokPerLane];
#pragma unroll
      for (int i = 0; i < kTokPerLane; ++i) {
        const uint16_t* tp = base + (int64_t)(lane + 32 * i) * row + 8 * c;
        kr[i] = ldg_stream16(tp);
        ki[i] = ldg_stream16(tp + a.F);
      }
      rope_chunk<G, E>(cf + 8 * c * CG, kr, ki, acc);
    }
    // partial RoPE: direct q_pass . k over the unrotated dims
#pragma unroll 1
    for (int c = 0; c < a.P / 8; ++c) {
      uint4 kp[kTokPerLane];
#pragma unroll
      for (int i = 0; i < kTokPerLane; ++i)
        kp[i] = ldg_stream16(base + (int64_t)(lane + 32 * i) * row + 2 * a.F + 8 * c);
      pass_chunk<G, E>(qp + 8 * c * G, kp, acc);
    }
    page_epilogue<G>(a, acc, lane, valid, l, h, p);
    __syncwarp();
  }
}

// --------------------------------------------------------------------------
// paged scorer (max over future offsets) -- the option's slow, exact path
// --------------------------------------------------------------------------

template <int G, class E>
__global__ void __launch_bounds__(kScoreWarps * 32) score_max_kernel(const __grid_constant__ ScoreArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  constexpr int CG = coef_group_stride(G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t units = (int64_t)a.L * a.total_pages * a.kvh;
  const int row = a.kvh * a.D;
  for (int64_t u = (int64_t)blockIdx.x * kScoreWarps + warp; u < units;
       u += (int64_t)gridDim.x * kScoreWarps) {
    const int h = u % a.kvh;
    const int p = (u / a.kvh) % a.total_pages;
    const int l = u / ((int64_t)a.kvh * a.total_pages);
    int r, valid;
    int64_t blk;
    if (!unit_page(a, p, r, valid, blk)) continue;
    const float* cf = a.coef + ((int64_t)(r * a.L + l) * a.kvh + h) * a.coef_block;
    const float* tab = cf + (int64_t)a.F * CG;
    const float* qpt = a.P ? a.q_pass_t + (int64_t)(l * a.kvh + h) * a.P * G : nullptr;
    const uint16_t* base = reinterpret_cast<const uint16_t*>(a.k_layers[l]) + blk * a.block_stride + (int64_t)h * a.D;
    float acc[kTokPerLane][G];
#pragma unroll
    for (int i = 0; i < kTokPerLane; ++i) {
      const uint16_t* tp = base + (int64_t)(lane + 32 * i) * row;
      float best[G], rest[G];
#pragma unroll
      for (int g = 0; g < G; ++g) { best[g] = -INFINITY; rest[g] = 0.f; }
      for (int o = 0; o < a.n_off; ++o) {
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
        for (int f = 0; f < a.F; ++f) {
          const float xr = unpack1(__ldg(tp + f), E{}), xi = unpack1(__ldg(tp + a.F + f), E{});
          const float* t2 = tab + ((int64_t)o * a.F + f) * 2 * G;
#pragma unroll
          for (int g = 0; g < G; ++g) s[g] = fmaf(xi, __ldg(t2 + G + g), fmaf(xr, __ldg(t2 + g), s[g]));
        }
#pragma unroll
        for (int g = 0; g < G; ++g) best[g] = nan_max(best[g], s[g]);
      }
      for (int f = 0; f < a.F; ++f) {
        const float xr = unpack1(__ldg(tp + f), E{}), xi = unpack1(__ldg(tp + a.F + f), E{});
        const float m = sqrtf(xr * xr + xi * xi);
#pragma unroll
        for (int g = 0; g < G; ++g) rest[g] = fmaf(m, __ldg(cf + f * CG + 2 * G + g), rest[g]);
      }
      for (int d = 0; d < a.P; ++d) {
        const float x = unpack1(__ldg(tp + 2 * a.F + d), E{});
#pragma unroll
        for (int g = 0; g < G; ++g) rest[g] = fmaf(x, __ldg(qpt + d * G + g), rest[g]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) acc[i][g] = best[g] + rest[g];
    }
    page_epilogue<G>(a, acc, lane, valid, l, h, p);
  }
}

// --------------------------------------------------------------------------
// per-head statistics
// --------------------------------------------------------------------------

// One CTA per (scoring layer, request).  The request's partials are the
// contiguous range [p0*parts, p1*parts) x heads of float2 (partial sum, sum of
// squared deviations from the partial's own mean).  Thread i owns head
// i % heads and every (blockDim / heads)-th partial of it, so a warp's loads
// are contiguous.  Two passes, both in fp64 and in a fixed order:
//   mean = (sum of the partial sums) / T
//   M2   = sum over partials of (M2_q + n_q * (mean_q - mean)^2)
// (the exact decomposition of the sum of squares about the overall mean), then
// var = M2 / T (population variance, as torch.var_mean(correction=0)).
__device__ __forceinline__ double reduce_slots(double v, double* red, int heads, int slots) {
  // sum of the `slots` per-thread values of each head (thread j * heads + h
  // holds slot j of head h) by a pairwise tree in a fixed order; returns it to
  // the slot-0 threads (threadIdx.x < heads)
  red[threadIdx.x] = v;
  __syncthreads();
  const int j = threadIdx.x / heads;
  int half = 1;
  while (half < slots) half <<= 1;
  for (half >>= 1; half >= 1; half >>= 1) {
    if (j < half && j + half < slots) red[threadIdx.x] += red[threadIdx.x + half * heads];
    __syncthreads();
  }
  const double s = red[threadIdx.x];
  __syncthreads();
  return s;
}

__global__ void __launch_bounds__(1024) head_stats_kernel(const float* __restrict__ partial, int L, int R,
                                                          int total_pages, int parts, int heads,
                                                          const int32_t* __restrict__ tokens,
                                                          const int32_t* __restrict__ page_off,
                                                          float* mean_out, float* var_out, float* den_out) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  extern __shared__ double red[];  // [blockDim]
  const int l = blockIdx.x, r = blockIdx.y;
  const int p0 = page_off[r], p1 = page_off[r + 1], T = tokens[r];
  const int span = kBlock / parts;  // tokens per partial
  (void)L;
  const int slots = blockDim.x / heads;  // threads per head
  const int h = threadIdx.x % heads, j = threadIdx.x / heads;
  const bool live = j < slots;
  const float2* part = reinterpret_cast<const float2*>(partial) + (int64_t)l * total_pages * parts * heads;
  const int q0 = p0 * parts;
  const int q1 = min(p1 * parts, q0 + (T + span - 1) / span);  // padding partials hold nothing
  constexpr int U = 8;  // partials whose loads are in flight together
  // one pass in fp64: S = sum of the partial sums, Q = sum over partials of
  // (M2_b + s_b^2 / n_b); then M2 = Q - S^2 / T (Chan's combination of all
  // partials about the overall mean, expanded)
  double s = 0.0, q2 = 0.0;
  if (live) {
    for (int q = q0 + j; q < q1; q += U * slots) {
      float2 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int qq = q + u * slots;
        v[u] = qq < q1 ? __ldg(part + (int64_t)qq * heads + h) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int qq = q + u * slots;
        if (qq < q1) {
          const int n = min(span, T - (qq - q0) * span);
          const double x = (double)v[u].x;
          s += x;
          q2 += (double)v[u].y + x * x / n;
        }
      }
    }
  }
  s = reduce_slots(live ? s : 0.0, red, heads, slots);
  q2 = reduce_slots(live ? q2 : 0.0, red, heads, slots);
  // valid in the first `heads` threads (reduce_slots returns there)
  const double mu = T > 0 ? s / T : 0.0;
  const double m2 = fmax(0.0, q2 - s * mu);
  if (threadIdx.x < heads) {
    const int64_t i = ((int64_t)l * R + r) * heads + threadIdx.x;
    const float var = T > 0 ? (float)(m2 / T) : NAN;
    mean_out[i] = T > 0 ? (float)mu : NAN;
    var_out[i] = var;
    den_out[i] = sqrtf(fmaxf(var, 1e-6f));
  }
}

// --------------------------------------------------------------------------
// normalisation, head max, layer aggregation
// --------------------------------------------------------------------------

// Grid (8-page blocks, scoring layers): one thread per (4 consecutive tokens,
// layer) computes the head max of the normalised scores (kvc_norm.cuh) and
// writes the layer's row; aggregate_rows then reduces the layers (TP = 1 and
// the NCCL sync).  Page padding is written as 0, keeping rows finite for the
// MAX sync.
// HS lanes share a token quad's heads (HS = 1: one lane takes all heads of 4
// tokens); a 256-thread CTA covers 256 / (32 * HS) pages.  Small batches use
// HS = 4 for four times the CTAs; large ones HS = 1 (less staging per page).
// agg: with a single scoring layer the layer aggregation is the identity, so
// the final score finalize(z) is written here too (null: rows only).
template <int HS>
__global__ void __launch_bounds__(256) normalize_kernel(const float* __restrict__ raw, int L, int heads,
                                                        int total_pages, const float* __restrict__ mean,
                                                        const float* __restrict__ den,
                                                        const int32_t* __restrict__ tokens,
                                                        const int32_t* __restrict__ page_off, int R,
                                                        float* rows, float* agg) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  constexpr int NP = 256 / (32 * HS);
  extern __shared__ float st[];  // [3][NP][heads]
  __shared__ NormPagesN<NP> np;
  const int l = blockIdx.y;
  const int page0 = blockIdx.x * NP;
  norm_stage_n<NP>(np, st, page0, l, heads, total_pages, R, tokens, page_off, mean, den);
  const int quad = threadIdx.x / HS, slice = threadIdx.x % HS;
  if (page0 + (quad >> 5) >= total_pages) return;  // warp-uniform: a warp's quads share a page
  int64_t tok;
  float4 z;
  norm_quad_split<NP, HS>(np, st, raw, l, heads, total_pages, page0, quad, slice, tok, z);
  if (slice != 0) return;
  *reinterpret_cast<float4*>(rows + (int64_t)l * total_pages * kBlock + tok) = z;
  if (agg)  // padding is 0 in z and stays 0
    *reinterpret_cast<float4*>(agg + tok) =
        make_float4(finalize_score(z.x), finalize_score(z.y), finalize_score(z.z), finalize_score(z.w));
}

__global__ void __launch_bounds__(256) aggregate_rows_kernel(const float* __restrict__ rows, int L,
                                                             int64_t tok_total,
                                                             const int32_t* __restrict__ tokens,
                                                             const int32_t* __restrict__ page_off, int R,
                                                             int layer_agg, float* agg) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  const int64_t first = (int64_t)blockIdx.x * blockDim.x;  // 256 tokens: two pages
  const int r_lo = request_of_page(page_off, R, (int)(first >> 7));
  const int r_hi = request_of_page(page_off, R, (int)((min64(first + blockDim.x, tok_total) - 1) >> 7));
  const int64_t tok = first + threadIdx.x;
  if (tok >= tok_total) return;
  const int p = (int)(tok >> 7);
  const int r = p == (int)(first >> 7) ? r_lo : r_hi;
  const int t = (int)(tok - (int64_t)__ldg(page_off + r) * kBlock);
  if (t >= __ldg(tokens + r)) {
    agg[tok] = 0.f;
    return;
  }
  float acc = rows[tok];
  for (int l = 1; l < L; ++l) {
    const float z = rows[(int64_t)l * tok_total + tok];
    acc = layer_agg == KVC_AGG_MEAN ? acc + z : nan_max(acc, z);
  }
  if (layer_agg == KVC_AGG_MEAN) acc = __fdiv_rn(acc, (float)L);
  agg[tok] = finalize_score(acc);
}

// --------------------------------------------------------------------------
// host launchers
// --------------------------------------------------------------------------

template <int G, class E>
int launch_score(const ScoreArgs& a, int aggregation, cudaStream_t st) {
  constexpr int CG = coef_group_stride(G);
  const int64_t units = (int64_t)a.L * a.total_pages * a.kvh;
  if (units == 0) return KVC_OK;
  const int64_t want = (units + kScoreWarps - 1) / kScoreWarps;
  const int grid = (int)min64(want, (int64_t)sm_count() * 16);
  if (aggregation == KVC_AGG_MEAN) {
    const size_t smem = (size_t)kScoreWarps * a.warp_floats * sizeof(float);
    static size_t configured[64] = {};  // per device (per-context attribute)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KVC_ECUDA;
    if (smem > 48 * 1024 && smem > configured[dev]) {
      if (cudaFuncSetAttribute(score_mean_kernel<G, E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem) != cudaSuccess)
        return KVC_ECUDA;
      configured[dev] = smem;
    }
    launch_dep(score_mean_kernel<G, E>, grid, dim3(kScoreWarps * 32), smem, st, a);
  } else {
    launch_dep(score_max_kernel<G, E>, grid, dim3(kScoreWarps * 32), 0, st, a);
  }
  (void)CG;
  return launch_status();
}

template <class E>
int dispatch_group(const ScoreArgs& a, int G, int aggregation, cudaStream_t st) {
  switch (G) {
    case 1: return launch_score<1, E>(a, aggregation, st);
    case 2: return launch_score<2, E>(a, aggregation, st);
    case 4: return launch_score<4, E>(a, aggregation, st);
    case 5: return launch_score<5, E>(a, aggregation, st);
    case 6: return launch_score<6, E>(a, aggregation, st);
    case 7: return launch_score<7, E>(a, aggregation, st);
    case 8: return launch_score<8, E>(a, aggregation, st);
    case 3: return launch_score<3, E>(a, aggregation, st);
    default: return KVC_EUNSUPPORTED;
  }
}

}  // namespace kvc

using namespace kvc;

extern "C" int64_t kvc_coef_floats(int num_freq, int group, int n_off, int aggregation) {
  if (num_freq <= 0 || group <= 0) return 0;
  int64_t n = (int64_t)num_freq * coef_group_stride(group);
  if (aggregation == KVC_AGG_MAX) n += (int64_t)n_off * num_freq * 2 * group;
  return n;
}

extern "C" int kvc_prepare_score_coefficients(const float* omega, const float* offsets, int n_off,
                                              const int64_t* round_start, int R, int L, int kvh,
                                              int G, int F, const float* q_real, const float* q_imag,
                                              const float* scale, const float* extra, int aggregation,
                                              float* coef_out, void* stream) {
  KVC_CHECK_ARG(omega && offsets && round_start && q_real && q_imag && scale && extra && coef_out, KVC_ENULL);
  KVC_CHECK_ARG(n_off > 0 && n_off <= 64 && R >= 0 && L > 0 && kvh > 0 && G > 0 && G <= 8 && F > 0 && F <= 256,
                KVC_EINVAL);
  KVC_CHECK_ARG(aggregation == KVC_AGG_MEAN || aggregation == KVC_AGG_MAX, KVC_EINVAL);
  if (R == 0) return KVC_OK;
  PrepArgs a{omega, offsets, round_start, q_real, q_imag, scale, extra, coef_out,
             n_off, R, L, kvh, G, F, aggregation, kvc_coef_floats(F, G, n_off, aggregation)};
  const size_t smem = (size_t)(2 * F + (aggregation == KVC_AGG_MAX ? 2 * n_off * F : 0)) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(prepare_coef_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return KVC_ECUDA;
  launch_dep(prepare_coef_kernel, dim3(L, R), dim3(256), smem, (cudaStream_t)stream, a);
  return launch_status();
}

extern "C" int kvc_score_paged_keys(const void* const* k_layers, int L, int dtype, int64_t block_stride,
                                    int64_t num_blocks, int kvh, int G, int D, int rot,
                                    const int64_t* src_blocks, const int64_t* src_block_off,
                                    const int32_t* tokens, const int32_t* page_off, int R, int total_pages,
                                    const float* coef, int n_off, int aggregation, const float* q_pass_t,
                                    float* raw_out, float* partial_out, int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(k_layers && src_blocks && src_block_off && tokens && page_off && coef && raw_out && partial_out,
                KVC_ENULL);
  KVC_CHECK_ARG(L > 0 && L <= kMaxLayers && kvh > 0 && G > 0 && D > 0 && rot > 0 && rot <= D && R >= 0 &&
                    total_pages >= 0 && num_blocks > 0 && n_off > 0,
                KVC_EINVAL);
  KVC_CHECK_ARG(dtype == KVC_BF16 || dtype == KVC_FP16, KVC_EINVAL);
  KVC_CHECK_ARG(aggregation == KVC_AGG_MEAN || aggregation == KVC_AGG_MAX, KVC_EINVAL);
  KVC_CHECK_ARG(block_stride >= (int64_t)kBlock * kvh * D, KVC_EINVAL);
  const int F = rot / 2, P = D - rot;
  KVC_CHECK_ARG(rot % 2 == 0, KVC_EINVAL);
  if (aggregation == KVC_AGG_MEAN) {
    // the streaming kernel reads 16-byte vectors of 8 elements
    KVC_CHECK_ARG(F % 8 == 0 && P % 8 == 0, KVC_EUNSUPPORTED);
    KVC_CHECK_ARG(block_stride % 8 == 0 && D % 8 == 0, KVC_EALIGN);
  }
  KVC_CHECK_ARG(P == 0 || q_pass_t != nullptr, KVC_ENULL);
  for (int l = 0; l < L; ++l) {
    KVC_CHECK_ARG(k_layers[l] != nullptr, KVC_ENULL);
    KVC_CHECK_ARG(aligned(k_layers[l], aggregation == KVC_AGG_MEAN ? 16 : 2), KVC_EALIGN);
  }
  KVC_CHECK_ARG(aligned(coef, 16) && (P == 0 || aligned(q_pass_t, 16)) && aligned(partial_out, 8), KVC_EALIGN);
  if (R == 0 || total_pages == 0) return KVC_OK;
  ScoreArgs a{};
  for (int l = 0; l < L; ++l) a.k_layers[l] = k_layers[l];
  a.block_stride = block_stride;
  a.num_blocks = num_blocks;
  a.src_blocks = src_blocks;
  a.src_block_off = src_block_off;
  a.tokens = tokens;
  a.page_off = page_off;
  a.coef = coef;
  a.q_pass_t = q_pass_t;
  a.raw = raw_out;
  a.partial = partial_out;
  a.error_flag = error_flag;
  a.coef_block = kvc_coef_floats(F, G, n_off, aggregation);
  a.tok_total = (int64_t)total_pages * kBlock;
  a.L = L;
  a.kvh = kvh;
  a.D = D;
  a.F = F;
  a.P = P;
  a.R = R;
  a.total_pages = total_pages;
  a.n_off = n_off;
  a.warp_floats = F * coef_group_stride(G) + P * G;
  a.warp_floats = (a.warp_floats + 3) & ~3;
  cudaStream_t st = (cudaStream_t)stream;
  return dtype == KVC_BF16 ? dispatch_group<Bf16>(a, G, aggregation, st) : dispatch_group<Fp16>(a, G, aggregation, st);
}

extern "C" int kvc_head_stats(const float* partial, int L, int R, int total_pages, int parts_per_page, int heads,
                              const int32_t* tokens, const int32_t* page_off, float* mean_out,
                              float* var_out, float* denom_out, void* stream) {
  KVC_CHECK_ARG(partial && tokens && page_off && mean_out && var_out && denom_out, KVC_ENULL);
  KVC_CHECK_ARG(L > 0 && R >= 0 && heads > 0 && total_pages >= 0, KVC_EINVAL);
  KVC_CHECK_ARG(parts_per_page > 0 && kBlock % parts_per_page == 0, KVC_EINVAL);
  if (R == 0) return KVC_OK;
  KVC_CHECK_ARG(heads <= 1024, KVC_EUNSUPPORTED);
  KVC_CHECK_ARG(R <= 65535, KVC_EINVAL);
  // the largest whole number of threads per head that fits 1024 threads
  const int threads = (1024 / heads) * heads;
  const int block = std::min(1024, ((threads + 31) / 32) * 32);
  launch_dep(head_stats_kernel, dim3(L, R), dim3(block), block * sizeof(double), (cudaStream_t)stream, partial, L, R,
             total_pages, parts_per_page, heads, tokens, page_off, mean_out, var_out, denom_out);
  return launch_status();
}

extern "C" int kvc_normalize_aggregate(const float* raw, int L, int heads, int total_pages, const float* mean,
                                       const float* denom, const int32_t* tokens, const int32_t* page_off,
                                       int R, int layer_aggregation, float* rows_out, float* agg_out,
                                       void* stream) {
  KVC_CHECK_ARG(raw && mean && denom && tokens && page_off && rows_out, KVC_ENULL);
  KVC_CHECK_ARG(L > 0 && L <= 65535 && heads > 0 && R >= 0 && total_pages >= 0, KVC_EINVAL);
  KVC_CHECK_ARG(layer_aggregation == KVC_AGG_MEAN || layer_aggregation == KVC_AGG_MAX, KVC_EINVAL);
  if (R == 0 || total_pages == 0) return KVC_OK;
  KVC_CHECK_ARG(aligned(raw, 16) && aligned(rows_out, 16), KVC_EALIGN);
  KVC_CHECK_ARG(agg_out == nullptr || aligned(agg_out, 16), KVC_EALIGN);
  // fewer than two CTAs per SM with 8 pages each: split the heads instead
  const bool split = (int64_t)((total_pages + 7) / 8) * L < 2 * (int64_t)sm_count();
  const int np = split ? 2 : 8;
  const dim3 grid((unsigned)((total_pages + np - 1) / np), (unsigned)L);
  const size_t smem = (size_t)3 * np * heads * sizeof(float);
  if (smem > 48 * 1024) return KVC_EUNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  const bool fused = agg_out != nullptr && L == 1;  // one layer: no separate layer reduction
  float* agg = fused ? agg_out : nullptr;
  if (split)
    launch_dep(normalize_kernel<4>, grid, dim3(256), smem, st, raw, L, heads, total_pages, mean, denom, tokens,
               page_off, R, rows_out, agg);
  else
    launch_dep(normalize_kernel<1>, grid, dim3(256), smem, st, raw, L, heads, total_pages, mean, denom, tokens,
               page_off, R, rows_out, agg);
  const int rc = launch_status();
  if (rc != KVC_OK || agg_out == nullptr || fused) return rc;
  return kvc_aggregate_rows(rows_out, L, total_pages, tokens, page_off, R, layer_aggregation, agg_out, stream);
}

extern "C" int kvc_aggregate_rows(const float* rows, int L, int total_pages, const int32_t* tokens,
                                  const int32_t* page_off, int R, int layer_aggregation, float* agg_out,
                                  void* stream) {
  KVC_CHECK_ARG(rows && tokens && page_off && agg_out, KVC_ENULL);
  KVC_CHECK_ARG(L > 0 && R >= 0 && total_pages >= 0, KVC_EINVAL);
  KVC_CHECK_ARG(layer_aggregation == KVC_AGG_MEAN || layer_aggregation == KVC_AGG_MAX, KVC_EINVAL);
  if (R == 0 || total_pages == 0) return KVC_OK;
  const int64_t tok_total = (int64_t)total_pages * kBlock;
  launch_dep(aggregate_rows_kernel, dim3((unsigned)((tok_total + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, rows,
             L, tok_total, tokens, page_off, R, layer_aggregation, agg_out);
  return launch_status();
}

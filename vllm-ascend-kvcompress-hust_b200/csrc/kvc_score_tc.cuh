// Pieces shared by the two tensor-core key scorers: the mma.sync kernel
// (kvc_score_tc.cu) and the tcgen05 kernel with TMEM accumulators
// (kvc_score_umma.cu).  Both evaluate, per (scoring layer, KV head, page),
//     Y[t, n] = sum_k X[t, k] * W[k, n]
//     X = [ kr | ki | m_hi | m_lo | k_pass ]      (m = sqrt(kr^2 + ki^2))
//     W = [ a  | b  |  e   | e_hi | q_pass ]      (a, b, e folded with the phases)
// with W's fp32 coefficients split into hi + lo 16-bit halves (columns n < 8:
// hi of query head n, n >= 8: lo of head n - 8) and m split likewise.
#pragma once

#include <cuda.h>

#include "kvc_async.cuh"

namespace kvc {

constexpr int kMaxTcLayers = 64;
constexpr int kBoxElems = 64;                      // 128-byte swizzle span of 16-bit elements
constexpr int kBoxBytes = kBoxElems * 2 * kBlock;  // one box: 128 tokens x 64 elements = 16 KB
constexpr int kTcQuarters = 4;                     // moments partials per page (32-token slices)

// 16-deep K steps of W: a, b, e, e_hi bands of F each, then the pass band
__host__ __device__ constexpr int frag_steps(int F, int P) { return 4 * (F / 16) + P / 16; }

// One (request, layer, head) record of W: frag_steps * 512 bytes of 16-bit
// values, then 16 bytes whose first float is the exact power of two that
// undoes W's scaling (w_scale); the scorers multiply their sums by it.
__host__ __device__ constexpr int64_t w_record_bytes(int F, int P) { return (int64_t)frag_steps(F, P) * 512 + 16; }

struct FragArgs {
  const float* omega;     // [L][F]
  const float* offsets;   // [n_off]
  const int64_t* round_start;
  const float* q_real;    // [L][kvh][G][F]
  const float* q_imag;
  const float* scale;
  const float* extra;
  const float* q_pass;    // [L][kvh][G][P] or null
  uint32_t* frag;         // per (request, layer, head): a record of w_record_bytes
  int n_off, R, L, kvh, G, F, P, half_fp16;
};

struct TcArgs {
  CUtensorMap maps[kMaxTcLayers];
  const int64_t* src_blocks;
  const int64_t* src_block_off;
  const int32_t* tokens;
  const int32_t* page_off;
  const uint4* frag;
  float* raw;
  float* partial;
  int32_t* error_flag;
  int64_t tok_total;
  int64_t num_blocks;
  int64_t units;        // layers_here * kvh * total_pages
  int layer0;           // global index of maps[0]
  int L_total;          // scoring layers (raw / partial / frag indexing)
  int kvh, G, R, total_pages;
};

__device__ __forceinline__ uint16_t to_half_bits(float v, int fp16) {
  if (fp16) {
    __half h = __float2half_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
  }
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}

__device__ __forceinline__ float from_half_bits(uint16_t v, int fp16) {
  return fp16 ? unpack1(v, Fp16{}) : unpack1(v, Bf16{});
}

// Shared-memory floats the W staging of one (layer, head) needs.
inline size_t w_stage_floats(int n_off, int F, int G) { return (size_t)(2 + 2 * n_off) * F + (size_t)4 * G * F; }

// Stage the inputs of W for (layer l, request r, KV head h) into `sm`
// (w_stage_floats): mean cos / sin of the phases over the offsets, and the
// head's q_real, q_imag, scale, extra.  All threads call it; ends synchronised.
__device__ __forceinline__ void stage_w_inputs(const FragArgs& a, float* sm, int l, int r, int h) {
  float* cm = sm;                      // [F] mean cos
  float* sn = sm + a.F;                // [F] mean sin
  float* tc = sm + 2 * a.F;            // [n_off][F] cos
  float* ts = tc + a.n_off * a.F;      // [n_off][F] sin
  float* qs = ts + a.n_off * a.F;      // [4][G][F] q_real, q_imag, scale, extra of this (layer, head)
  const float rs = (float)a.round_start[r];
  {
    const int gf = a.G * a.F;
    const int64_t base = (int64_t)(l * a.kvh + h) * gf;
    for (int i = threadIdx.x; i < gf; i += blockDim.x) {
      qs[i] = a.q_real[base + i];
      qs[gf + i] = a.q_imag[base + i];
      qs[2 * gf + i] = a.scale[base + i];
      qs[3 * gf + i] = a.extra[base + i];
    }
  }
  for (int i = threadIdx.x; i < a.n_off * a.F; i += blockDim.x) {
    const int o = i / a.F, f = i % a.F;
    // fp32 (offset + round_start) then * omega, as the reference forms phases
    const float ph = __fmul_rn(__fadd_rn(a.offsets[o], rs), a.omega[l * a.F + f]);
    sincosf(ph, &ts[i], &tc[i]);
  }
  __syncthreads();
  for (int f = threadIdx.x; f < a.F; f += blockDim.x) {
    float cs = 0.f, ss = 0.f;
    for (int o = 0; o < a.n_off; ++o) {  // offsets summed in order
      cs += tc[o * a.F + f];
      ss += ts[o * a.F + f];
    }
    const float inv = 1.0f / (float)a.n_off;
    cm[f] = cs * inv;
    sn[f] = ss * inv;
  }
  __syncthreads();
}

// W[k, g] for query head g < G and 0 <= k < 4F + P (stage_w_inputs staged).
// lo_zero: only the hi half is used (the m_lo band pairs with e_hi).
__device__ __forceinline__ float w_value(const FragArgs& a, const float* sm, int l, int h, int g, int k,
                                         bool& lo_zero) {
  const float* cm = sm;
  const float* sn = sm + a.F;
  const float* qs = sm + (2 + 2 * a.n_off) * a.F;
  const int gf = a.G * a.F;
  lo_zero = false;
  const int part = k / a.F;  // 0 a, 1 b, 2 e, 3 e (m_lo), >= 4 pass
  if (part < 4) {
    const int f = k - part * a.F;
    const int src = g * a.F + f;
    const float qr = qs[src], qi = qs[gf + src], sc = qs[2 * gf + src];
    if (part == 0) return sc * (qr * cm[f] - qi * sn[f]);
    if (part == 1) return sc * (qi * cm[f] + qr * sn[f]);
    lo_zero = part == 3;
    return qs[3 * gf + src] * sc;
  }
  const int p = k - 4 * a.F;
  return a.q_pass[((int64_t)(l * a.kvh + h) * a.G + g) * a.P + p];
}

// Power of two applied to W of (layer l, head h) before its 16-bit hi/lo
// split.  fp16 has a narrow exponent range: coefficients of low-|q| heads
// (1e-4 .. 1e-6) would fall into its subnormals and lose the lo half, so W
// is scaled until its largest magnitude lies in [2^13, 2^14).  bf16 keeps
// fp32's range and takes scale 1.  All threads call it (it synchronises).
__device__ __forceinline__ float w_scale(const FragArgs& a, const float* sm, int l, int h, float* red) {
  if (!a.half_fp16) return 1.f;
  const int kw = 4 * a.F + a.P;
  float m = 0.f;
  for (int i = threadIdx.x; i < a.G * kw; i += blockDim.x) {
    bool lo_zero;
    m = fmaxf(m, fabsf(w_value(a, sm, l, h, i / kw, i % kw, lo_zero)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  if (!(m > 0.f) || !isfinite(m)) return 1.f;
  int e;
  frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1)
  return ldexpf(1.f, max(-100, min(100, 14 - e)));
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, Bf16) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi, Fp16) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// kr^2 + ki^2 in fp32 for the two 16-bit halves of a word pair: mixed-precision
// FMAs square the 16-bit values directly (exact in fp32) and round the sum once,
// as fp32 arithmetic on the widened values would.
__device__ __forceinline__ float2 sum_squares2(uint32_t kr, uint32_t ki, Bf16) {
  float s0, s1;
  asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %2;\n\tmov.b32 {b0, b1}, %3;\n\t"
      "fma.rn.f32.bf16 %0, a0, a0, 0f00000000;\n\tfma.rn.f32.bf16 %0, b0, b0, %0;\n\t"
      "fma.rn.f32.bf16 %1, a1, a1, 0f00000000;\n\tfma.rn.f32.bf16 %1, b1, b1, %1;\n\t}"
      : "=f"(s0), "=f"(s1)
      : "r"(kr), "r"(ki));
  return make_float2(s0, s1);
}
__device__ __forceinline__ float2 sum_squares2(uint32_t kr, uint32_t ki, Fp16) {
  float s0, s1;
  asm("{\n\t.reg .b16 a0, a1, b0, b1;\n\tmov.b32 {a0, a1}, %2;\n\tmov.b32 {b0, b1}, %3;\n\t"
      "fma.rn.f32.f16 %0, a0, a0, 0f00000000;\n\tfma.rn.f32.f16 %0, b0, b0, %0;\n\t"
      "fma.rn.f32.f16 %1, a1, a1, 0f00000000;\n\tfma.rn.f32.f16 %1, b1, b1, %1;\n\t}"
      : "=f"(s0), "=f"(s1)
      : "r"(kr), "r"(ki));
  return make_float2(s0, s1);
}

// m = |(kr, ki)| for 8 packed elements, split into hi + lo halves
template <class E>
__device__ __forceinline__ void modulus_split(const uint32_t* kr, const uint32_t* ki, uint32_t* hi, uint32_t* lo) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 sq = sum_squares2(kr[i], ki[i], E{});
    const float2 mod = make_float2(sqrt_approx(sq.x), sqrt_approx(sq.y));
    hi[i] = pack2(mod.x, mod.y, E{});
    const float2 h = unpack2(hi[i], E{});
    const float2 d = __ffma2_rn(h, make_float2(-1.f, -1.f), mod);
    lo[i] = pack2(d.x, d.y, E{});
  }
}

// The tcgen05 scorer (kvc_score_umma.cu) serves these (rotary/2, pass)
// geometries; its W layout (prepare_w_umma) differs from the mma.sync
// fragments, so prepare and score both choose by this predicate.
bool umma_geometry(int F, int P);
int prepare_w_umma(const FragArgs& a, cudaStream_t st);
int launch_umma(const TcArgs& a, int F, int P, bool fp16, cudaStream_t st);

}  // namespace kvc

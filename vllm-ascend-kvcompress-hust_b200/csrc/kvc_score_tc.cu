// Tensor-core trigonometric key scorer for sm_100a: TMA-staged pages, bf16 MMA.
//
// Per (scoring layer l, KV head h, request r) the raw score of every cached key
// is a small matrix product: for the 128 tokens of a page
//     Y[t, g] = sum_k X[t, k] * W[k, g]
//     X = [ kr | ki | m_hi | m_lo | k_pass ]      (m = sqrt(kr^2 + ki^2))
//     W = [ a  | b  |  e   |  e   | q_pass ]      (a, b, e folded with the phases)
// Keys are exact in bf16 (they are bf16 in the cache); the fp32 coefficients
// are split into hi + lo bf16 parts held in the two 8-column halves of a
// 16-column B operand (Y[:, g] = C[:, g] + C[:, 8 + g]), and m into
// m_hi + m_lo; the dropped m_lo * e_lo term is ~2^-18 relative.  The MMA
// accumulates in fp32.  This keeps fp32-level agreement with the reference's
// fp32 scorer at a fraction of the CUDA-core instruction count.
//
// Data path: a producer warp streams each (page, head) K tile (128 tokens x
// head_dim) from the paged cache with cp.async.bulk.tensor (4-D tensor map
// over [blocks][128][kv_heads][head_dim], 64-element boxes, 128-byte swizzle)
// into a ring of shared-memory stages guarded by mbarriers; four consumer
// warps each own 32 tokens (two m16 tiles), load A fragments with ldmatrix
// (conflict-free on the swizzled layout), compute m in registers from the kr/ki
// fragments, and issue mma.sync.m16n8k16.  Every wait is bounded by a
// global-timer deadline; on expiry the kernel raises KVC_DEV_TIMEOUT and exits.
//
// The B-operand fragments of W are produced once per (request, layer, head) by
// prepare_frag_kernel directly in the per-lane register layout, so a consumer
// loads them with 16-byte coalesced loads when its unit's (r, l, h) changes.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "kvc_score_tc.cuh"

namespace kvc {

constexpr int kTcConsumers = 4;
constexpr int kTcThreads = (kTcConsumers + 1) * 32;
static_assert(kTcConsumers == kTcQuarters, "one moments partial per consumer warp");

// ---------------------------------------------------------------------------
// B-operand fragments of W (prepared once per (request, layer, head))
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) prepare_frag_kernel(const __grid_constant__ FragArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  extern __shared__ float sm[];
  const int l = blockIdx.x, r = blockIdx.y, h = blockIdx.z;
  __shared__ float red[8];
  stage_w_inputs(a, sm, l, r, h);
  const float scale = w_scale(a, sm, l, h, red);
  const int S = frag_steps(a.F, a.P);
  // this (request, layer, head)'s record: S*32 uint4 of fragments, then the inverse scale
  uint4* rec = reinterpret_cast<uint4*>(a.frag) + ((int64_t)(r * a.L + l) * a.kvh + h) * (S * 32 + 1);
  if (threadIdx.x == 0) rec[S * 32] = make_uint4(__float_as_uint(1.f / scale), 0u, 0u, 0u);
  for (int i = threadIdx.x; i < S * 32; i += blockDim.x) {
    const int lane = i % 32;
    const int s = i / 32;
    uint32_t words[4];
    for (int t = 0; t < 2; ++t) {          // n-tile: 0 = hi columns, 1 = lo columns
      const int g = lane / 4;              // column within the n-tile = query head
      for (int q = 0; q < 2; ++q) {        // register: k rows 0..7 / 8..15 of the step
        uint32_t word = 0;
        for (int e = 0; e < 2; ++e) {
          const int k = 16 * s + 2 * (lane % 4) + 8 * q + e;  // K index of W
          bool lo_zero = false;
          const float v = g < a.G ? w_value(a, sm, l, h, g, k, lo_zero) * scale : 0.f;
          const uint16_t hi = to_half_bits(v, a.half_fp16);
          uint16_t bits;
          if (t == 0) bits = hi;
          else bits = lo_zero ? 0 : to_half_bits(v - from_half_bits(hi, a.half_fp16), a.half_fp16);
          word |= (uint32_t)bits << (16 * e);
        }
        words[2 * t + q] = word;
      }
    }
    rec[s * 32 + lane] = make_uint4(words[0], words[1], words[2], words[3]);
  }
}

// ---------------------------------------------------------------------------
// PTX helpers (mbarrier, TMA, ldmatrix, mma)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

template <class E>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<Bf16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<Fp16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// the scorer
// ---------------------------------------------------------------------------

template <int F, int P>
struct TcGeom {
  static constexpr int D = 2 * F + P;
  static constexpr int S = frag_steps(F, P);
  static constexpr int kBoxes = D / kBoxElems;
  static constexpr int kStageBytes = kBoxes * kBoxBytes;
  static constexpr int kWBytes = S * 32 * 16;  // B fragments of one (request, layer, head)
  static constexpr int kStages = D <= 64 ? 3 : D <= 128 ? 2 : 3;
  static constexpr int kMinBlocks = D <= 128 ? 3 : 1;
  // stages | W buffer | full/empty/wfull/wfree barriers | unit metadata
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kWBytes + 8 * (2 * kStages + 2) + 32 * kStages;
};

// Shared-memory byte address of 16-element column group `col16` (dims col16*16 ..)
// of the 16-row tile starting at `row0`, for this lane's ldmatrix.x4 row.
__device__ __forceinline__ uint32_t frag_addr(uint32_t stage, int row0, int dim0, int lane) {
  const int row = row0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int dim = dim0 + (lane >> 4) * 8;
  const int box = dim / kBoxElems;
  const int chunk = (dim % kBoxElems) / 8;
  return stage + box * kBoxBytes + row * 128 + ((chunk ^ (row & 7)) << 4);
}

// Unit metadata the producer hands to the consumers with each stage.
struct UnitMeta {
  int p, h, lg, valid, wgen, end;
  float scale;  // undoes the W scaling of the unit's (request, layer, head)
};
static_assert(sizeof(UnitMeta) <= 32, "32 bytes of metadata per stage");

// Pipeline (per CTA): one producer lane resolves its contiguous range of
// (layer, head, page) units, publishes each unit's metadata and issues the
// page's TMA boxes into a ring stage (full/empty mbarriers).  The B-operand
// fragments W of the unit's (request, layer, head) live in one shared buffer:
// when they change ("generation" n), the producer first publishes the stage,
// then waits until every consumer warp has released generation n-1 (wfree),
// and bulk-copies the new fragments (wfull).  Consumers thus never hold W in
// registers, which leaves room for three CTAs per SM.
template <int F, int P, class E>
__global__ void __launch_bounds__(kTcThreads, TcGeom<F, P>::kMinBlocks) score_tc_kernel(const __grid_constant__ TcArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  using Gm = TcGeom<F, P>;
  constexpr int KF = F / 16;
  constexpr int KP = P / 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint4* wsm = reinterpret_cast<const uint4*>(base + Gm::kStages * Gm::kStageBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + Gm::kStages * Gm::kStageBytes + Gm::kWBytes);
  UnitMeta* meta = reinterpret_cast<UnitMeta*>(bars + 2 * Gm::kStages + 2);
  const uint32_t stage0 = smem_u32(base);
  const uint32_t wbuf = smem_u32(wsm);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + Gm::kStages);
  const uint32_t wfull = smem_u32(bars + 2 * Gm::kStages), wfree = wfull + 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Gm::kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kTcConsumers);
    }
    mbar_init(wfull, 1);
    mbar_init(wfree, kTcConsumers);
    mbar_init_fence();
  }
  __syncthreads();
  const int heads = a.kvh * a.G;

  if (warp == kTcConsumers) {
    // ---------------- producer -------------------------------------------------
    if (lane != 0) return;
    const int64_t per = (a.units + gridDim.x - 1) / gridDim.x;
    const int64_t u0 = (int64_t)blockIdx.x * per;
    const int64_t u1 = min64(a.units, u0 + per);
    uint32_t it = 0;
    int r = 0, cur_key = -1, gen = -1;
    float wscale = 1.f;
    bool ok = true;
    for (int64_t u = u0; u < u1 && ok; ++u) {
      const int p = (int)(u % a.total_pages);
      const int h = (int)((u / a.total_pages) % a.kvh);
      const int l = (int)(u / ((int64_t)a.total_pages * a.kvh));
      if (u == u0 || p == 0) r = request_of_page(a.page_off, a.R, p);
      while (__ldg(a.page_off + r + 1) <= p) ++r;  // units advance page by page
      const int pl = p - __ldg(a.page_off + r);
      const int64_t blk = __ldg(a.src_blocks + __ldg(a.src_block_off + r) + pl);
      if (blk < 0 || blk >= a.num_blocks) {
        raise_flag(a.error_flag, KVC_DEV_BLOCK_RANGE);
        continue;
      }
      const int lg = a.layer0 + l;
      const int key = (r * a.L_total + lg) * a.kvh + h;
      const bool new_w = key != cur_key;
      if (new_w) {
        cur_key = key;
        ++gen;
        wscale = __ldg(reinterpret_cast<const float*>(a.frag + (int64_t)key * (Gm::S * 32 + 1) + Gm::S * 32));
      }
      const int s = it % Gm::kStages;
      if (!mbar_wait(empty0 + 8 * s, ((it / Gm::kStages) & 1) ^ 1, a.error_flag)) {
        ok = false;
        break;
      }
      meta[s] = UnitMeta{p, h, lg, min(kBlock, __ldg(a.tokens + r) - pl * kBlock), gen, 0, wscale};
      mbar_expect_tx(full0 + 8 * s, Gm::kStageBytes);
#pragma unroll
      for (int b = 0; b < Gm::kBoxes; ++b)
        tma_load_4d(stage0 + s * Gm::kStageBytes + b * kBoxBytes, &a.maps[l], b * kBoxElems, h, 0, (int)blk,
                    full0 + 8 * s);
      ++it;
      if (new_w) {
        // the consumers release generation gen-1 when they reach this stage
        if (gen > 0 && !mbar_wait(wfree, (gen - 1) & 1, a.error_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(wfull, Gm::kWBytes);
        bulk_load(wbuf, a.frag + (int64_t)key * (Gm::S * 32 + 1), Gm::kWBytes, wfull);
      }
    }
    if (ok) {  // sentinel stage: tells the consumers the range is done
      const int s = it % Gm::kStages;
      if (mbar_wait(empty0 + 8 * s, ((it / Gm::kStages) & 1) ^ 1, a.error_flag)) {
        meta[s].end = 1;
        mbar_arrive(full0 + 8 * s);
        ++it;
      }
    }
    // drain: every issued copy must have landed before the CTA may exit
    for (uint32_t k = 0; k < Gm::kStages && k < it; ++k) {
      const uint32_t j = it - 1 - k;
      mbar_wait(full0 + 8 * (j % Gm::kStages), (j / Gm::kStages) & 1, a.error_flag);
    }
    if (gen >= 0) mbar_wait(wfull, gen & 1, a.error_flag);
    return;
  }

  // ---------------- consumers: 4 warps x 32 tokens of each 128-token tile ----
  int cur_gen = -1;
  // per-lane byte offsets of the ldmatrix rows of this warp's two m16 tiles
  for (uint32_t it = 0;; ++it) {
    const int s = it % Gm::kStages;
    // waits are voted warp-wide, so a timed-out warp leaves as a whole (the
    // epilogue's shuffles name every lane)
    if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8 * s, (it / Gm::kStages) & 1, a.error_flag))) return;
    const UnitMeta mu = meta[s];
    if (mu.end) break;
    if (mu.wgen != cur_gen) {
      __syncwarp();
      if (cur_gen >= 0 && lane == 0) mbar_arrive(wfree);  // done with the previous fragments
      if (!__all_sync(0xffffffffu, mbar_wait(wfull, mu.wgen & 1, a.error_flag))) return;
      cur_gen = mu.wgen;
    }
    const uint32_t stage = stage0 + s * Gm::kStageBytes;
    const uint4* wl = wsm + lane;

    // accumulators per 16-token tile mt: kr/ki products in the hi / lo column
    // halves (c0, c1), modulus products likewise (c2, c3); the pass band adds
    // to c0 / c1.  W fragments are loaded once per K step for both tiles.
    float c0[2][4] = {}, c1[2][4] = {}, c2[2][4] = {}, c3[2][4] = {};
#pragma unroll
    for (int j = 0; j < KF; ++j) {
      const uint4 wa = wl[j * 32], wb = wl[(KF + j) * 32];
      const uint4 we = wl[(2 * KF + j) * 32], wf = wl[(3 * KF + j) * 32];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int row0 = warp * 32 + mt * 16;
        uint32_t kr[4], ki[4], mh[4], ml[4];
        ldsm_x4(frag_addr(stage, row0, 16 * j, lane), kr);
        ldsm_x4(frag_addr(stage, row0, F + 16 * j, lane), ki);
        mma16816<E>(c0[mt], kr, wa.x, wa.y);
        mma16816<E>(c1[mt], kr, wa.z, wa.w);
        mma16816<E>(c0[mt], ki, wb.x, wb.y);
        mma16816<E>(c1[mt], ki, wb.z, wb.w);
        modulus_split<E>(kr, ki, mh, ml);
        mma16816<E>(c2[mt], mh, we.x, we.y);
        mma16816<E>(c3[mt], mh, we.z, we.w);
        mma16816<E>(c2[mt], ml, wf.x, wf.y);
      }
    }
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const uint4 wp = wl[(4 * KF + j) * 32];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t kp[4];
        ldsm_x4(frag_addr(stage, warp * 32 + mt * 16, 2 * F + 16 * j, lane), kp);
        mma16816<E>(c0[mt], kp, wp.x, wp.y);
        mma16816<E>(c1[mt], kp, wp.z, wp.w);
      }
    }
    float y[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) y[mt][i] = (c0[mt][i] + c1[mt][i]) + (c2[mt][i] + c3[mt][i]);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);

    // ---- epilogue: raw scores and the quarter-page moments of each query head
    // lane holds heads g = 2*(lane%4) + {0,1} for tokens warp*32 + {0,8,16,24} + lane/4
    const int nq = max(0, min(32, mu.valid - warp * 32));
    const float inv_nq = nq > 0 ? __frcp_rn((float)nq) : 0.f;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int g = 2 * (lane & 3) + gi;
      float vals[4];
      bool ok[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = warp * 32 + (i >> 1) * 16 + (i & 1) * 8 + (lane >> 2);
        vals[i] = y[i >> 1][(i & 1) * 2 + gi] * mu.scale;  // exact: a power of two
        ok[i] = t < mu.valid && g < a.G;
      }
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) sum += ok[i] ? vals[i] : 0.f;
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      // centring value for M2 only: any value near the mean keeps Chan's combination exact
      const float mean = sum * inv_nq;
      float m2 = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float d = vals[i] - mean;
        m2 += ok[i] ? d * d : 0.f;
      }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) m2 += __shfl_xor_sync(0xffffffffu, m2, o);
      if (g < a.G) {
        float* row = a.raw + (((int64_t)mu.lg * a.total_pages + mu.p) * heads + mu.h * a.G + g) * kBlock;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = warp * 32 + (i >> 1) * 16 + (i & 1) * 8 + (lane >> 2);
          if (ok[i]) row[t] = vals[i];
        }
        if (lane < 4) {
          float2* out = reinterpret_cast<float2*>(a.partial) +
                        (((int64_t)mu.lg * a.total_pages + mu.p) * 4 + warp) * heads + mu.h * a.G + g;
          *out = make_float2(sum, m2);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

template <int F, int P, class E>
int launch_tc(const TcArgs& a, cudaStream_t st) {
  using Gm = TcGeom<F, P>;
  if (a.units == 0) return KVC_OK;
  static bool configured[64] = {};  // per device: the shared-memory opt-in is a per-context attribute
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KVC_ECUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(score_tc_kernel<F, P, E>, cudaFuncAttributeMaxDynamicSharedMemorySize, Gm::kSmem) !=
        cudaSuccess)
      return KVC_ECUDA;
    configured[dev] = true;
  }
  const int64_t cap = (int64_t)sm_count() * Gm::kMinBlocks;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cap, a.units));
  launch_dep(score_tc_kernel<F, P, E>, dim3(grid), dim3(kTcThreads), Gm::kSmem, st, a);
  return launch_status();
}

template <class E>
int dispatch_tc(const TcArgs& a, int F, int P, cudaStream_t st) {
  if (F == 64 && P == 0) return launch_tc<64, 0, E>(a, st);
  if (F == 32 && P == 0) return launch_tc<32, 0, E>(a, st);
  if (F == 32 && P == 192) return launch_tc<32, 192, E>(a, st);
  if (F == 32 && P == 64) return launch_tc<32, 64, E>(a, st);
  if (F == 64 && P == 128) return launch_tc<64, 128, E>(a, st);
  if (F == 128 && P == 0) return launch_tc<128, 0, E>(a, st);
  return KVC_EUNSUPPORTED;
}

bool tc_geometry_supported(int G, int D, int rot) {
  const int F = rot / 2, P = D - rot;
  if (G < 1 || G > 8 || rot % 2) return false;
  return (F == 64 && P == 0) || (F == 32 && P == 0) || (F == 32 && P == 192) || (F == 32 && P == 64) ||
         (F == 64 && P == 128) || (F == 128 && P == 0);
}

}  // namespace kvc

using namespace kvc;

extern "C" int kvc_tc_supported(int group, int head_dim, int rotary_dim) {
  return tc_geometry_supported(group, head_dim, rotary_dim) ? 1 : 0;
}

extern "C" int kvc_tc05_supported(int group, int head_dim, int rotary_dim) {
  const bool ok = group >= 1 && group <= 8 && rotary_dim % 2 == 0 && head_dim >= rotary_dim &&
                  umma_geometry(rotary_dim / 2, head_dim - rotary_dim);
  return ok ? 1 : 0;
}

// One moments partial per 32-token slice of a page (both tensor-core scorers).
extern "C" int kvc_tc_partials_per_page(void) { return kTcQuarters; }

extern "C" int64_t kvc_fragment_words(int num_freq, int pass_dim) {
  if (num_freq <= 0 || num_freq % 16 || pass_dim < 0 || pass_dim % 16) return 0;
  return w_record_bytes(num_freq, pass_dim) / 4;
}

extern "C" int kvc_encode_key_maps(const void* const* k_layers, int L, int dtype, int64_t block_stride,
                                   int64_t num_blocks, int kvh, int D, void* maps_out) {
  KVC_CHECK_ARG(k_layers && maps_out, KVC_ENULL);
  KVC_CHECK_ARG(L > 0 && kvh > 0 && D > 0 && num_blocks > 0 && (dtype == KVC_BF16 || dtype == KVC_FP16),
                KVC_EINVAL);
  KVC_CHECK_ARG(D % kBoxElems == 0, KVC_EUNSUPPORTED);
  KVC_CHECK_ARG(block_stride >= (int64_t)kBlock * kvh * D && (block_stride * 2) % 16 == 0, KVC_EALIGN);
  PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return KVC_ECUDA;
  unsigned char* out = reinterpret_cast<unsigned char*>(maps_out);  // caller's buffer: any alignment
  for (int l = 0; l < L; ++l) {
    KVC_CHECK_ARG(k_layers[l] != nullptr, KVC_ENULL);
    KVC_CHECK_ARG(aligned(k_layers[l], 16), KVC_EALIGN);
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)kvh, (cuuint64_t)kBlock, (cuuint64_t)num_blocks};
    const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)kvh * D * 2, (cuuint64_t)block_stride * 2};
    const cuuint32_t box[4] = {kBoxElems, 1, kBlock, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUtensorMap tmp;
    const CUresult rc = fn(&tmp, dtype == KVC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                           4, const_cast<void*>(k_layers[l]), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) return KVC_EINVAL;
    memcpy(out + (size_t)l * sizeof(CUtensorMap), &tmp, sizeof(CUtensorMap));
  }
  return KVC_OK;
}

// W for either tensor-core scorer: mma.sync register fragments, or (umma) the
// swizzled shared-memory matrix the tcgen05 scorer's descriptors read.
static int prepare_fragments(bool umma, const float* omega, const float* offsets, int n_off,
                             const int64_t* round_start, int R, int L, int kvh, int G, int F, int P,
                             const float* q_real, const float* q_imag, const float* scale, const float* extra,
                             const float* q_pass, int dtype, uint32_t* frag_out, void* stream) {
  KVC_CHECK_ARG(omega && offsets && round_start && q_real && q_imag && scale && extra && frag_out, KVC_ENULL);
  KVC_CHECK_ARG(n_off > 0 && n_off <= 64 && R >= 0 && L > 0 && kvh > 0 && G > 0 && G <= 8, KVC_EINVAL);
  KVC_CHECK_ARG(F > 0 && F % 16 == 0 && P >= 0 && P % 16 == 0, KVC_EUNSUPPORTED);
  KVC_CHECK_ARG(P == 0 || q_pass != nullptr, KVC_ENULL);
  KVC_CHECK_ARG(dtype == KVC_BF16 || dtype == KVC_FP16, KVC_EINVAL);
  KVC_CHECK_ARG(aligned(frag_out, 16), KVC_EALIGN);
  if (R == 0) return KVC_OK;
  FragArgs a{omega, offsets, round_start, q_real, q_imag, scale, extra, q_pass, frag_out,
             n_off, R, L, kvh, G, F, P, dtype == KVC_FP16 ? 1 : 0};
  const size_t smem = w_stage_floats(n_off, F, G) * sizeof(float);
  KVC_CHECK_ARG(smem <= 48 * 1024, KVC_EUNSUPPORTED);
  if (umma) {
    KVC_CHECK_ARG(umma_geometry(F, P), KVC_EUNSUPPORTED);
    return prepare_w_umma(a, (cudaStream_t)stream);
  }
  launch_dep(prepare_frag_kernel, dim3(L, R, kvh), dim3(256), smem, (cudaStream_t)stream, a);
  return launch_status();
}

extern "C" int kvc_prepare_score_fragments(const float* omega, const float* offsets, int n_off,
                                           const int64_t* round_start, int R, int L, int kvh, int G, int F, int P,
                                           const float* q_real, const float* q_imag, const float* scale,
                                           const float* extra, const float* q_pass, int dtype, uint32_t* frag_out,
                                           void* stream) {
  return prepare_fragments(false, omega, offsets, n_off, round_start, R, L, kvh, G, F, P, q_real, q_imag, scale,
                           extra, q_pass, dtype, frag_out, stream);
}

extern "C" int kvc_prepare_score_fragments_tc05(const float* omega, const float* offsets, int n_off,
                                                const int64_t* round_start, int R, int L, int kvh, int G, int F,
                                                int P, const float* q_real, const float* q_imag, const float* scale,
                                                const float* extra, const float* q_pass, int dtype,
                                                uint32_t* frag_out, void* stream) {
  return prepare_fragments(true, omega, offsets, n_off, round_start, R, L, kvh, G, F, P, q_real, q_imag, scale,
                           extra, q_pass, dtype, frag_out, stream);
}

static int score_tc(bool umma, const void* key_maps, int L, int dtype, int64_t num_blocks, int kvh, int G, int D,
                    int rot, const int64_t* src_blocks, const int64_t* src_block_off, const int32_t* tokens,
                    const int32_t* page_off, int R, int total_pages, const uint32_t* frag, float* raw_out,
                    float* partial_out, int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(key_maps && src_blocks && src_block_off && tokens && page_off && frag && raw_out && partial_out,
                KVC_ENULL);
  KVC_CHECK_ARG(L > 0 && kvh > 0 && R >= 0 && total_pages >= 0 && num_blocks > 0, KVC_EINVAL);
  KVC_CHECK_ARG(dtype == KVC_BF16 || dtype == KVC_FP16, KVC_EINVAL);
  KVC_CHECK_ARG(umma ? G >= 1 && G <= 8 && rot % 2 == 0 && umma_geometry(rot / 2, D - rot)
                     : tc_geometry_supported(G, D, rot),
                KVC_EUNSUPPORTED);
  KVC_CHECK_ARG(aligned(frag, 16) && aligned(partial_out, 8), KVC_EALIGN);
  if (R == 0 || total_pages == 0) return KVC_OK;
  const unsigned char* maps = reinterpret_cast<const unsigned char*>(key_maps);
  cudaStream_t st = (cudaStream_t)stream;
  for (int l0 = 0; l0 < L; l0 += kMaxTcLayers) {
    TcArgs a{};
    const int nl = std::min(kMaxTcLayers, L - l0);
    memcpy(a.maps, maps + (size_t)l0 * sizeof(CUtensorMap), sizeof(CUtensorMap) * nl);
    a.src_blocks = src_blocks;
    a.src_block_off = src_block_off;
    a.tokens = tokens;
    a.page_off = page_off;
    a.frag = reinterpret_cast<const uint4*>(frag);
    a.raw = raw_out;
    a.partial = partial_out;
    a.error_flag = error_flag;
    a.tok_total = (int64_t)total_pages * kBlock;
    a.num_blocks = num_blocks;
    a.units = (int64_t)nl * kvh * total_pages;
    a.layer0 = l0;
    a.L_total = L;
    a.kvh = kvh;
    a.G = G;
    a.R = R;
    a.total_pages = total_pages;
    const int F = rot / 2, P = D - rot;
    const int rc = umma                ? launch_umma(a, F, P, dtype == KVC_FP16, st)
                   : dtype == KVC_BF16 ? dispatch_tc<Bf16>(a, F, P, st)
                                       : dispatch_tc<Fp16>(a, F, P, st);
    if (rc != KVC_OK) return rc;
  }
  return KVC_OK;
}

extern "C" int kvc_score_paged_keys_tc(const void* key_maps, int L, int dtype, int64_t num_blocks, int kvh, int G,
                                       int D, int rot, const int64_t* src_blocks, const int64_t* src_block_off,
                                       const int32_t* tokens, const int32_t* page_off, int R, int total_pages,
                                       const uint32_t* frag, float* raw_out, float* partial_out,
                                       int32_t* error_flag, void* stream) {
  return score_tc(false, key_maps, L, dtype, num_blocks, kvh, G, D, rot, src_blocks, src_block_off, tokens, page_off,
                  R, total_pages, frag, raw_out, partial_out, error_flag, stream);
}

extern "C" int kvc_score_paged_keys_tc05(const void* key_maps, int L, int dtype, int64_t num_blocks, int kvh, int G,
                                         int D, int rot, const int64_t* src_blocks, const int64_t* src_block_off,
                                         const int32_t* tokens, const int32_t* page_off, int R, int total_pages,
                                         const uint32_t* frag, float* raw_out, float* partial_out,
                                         int32_t* error_flag, void* stream) {
  return score_tc(true, key_maps, L, dtype, num_blocks, kvh, G, D, rot, src_blocks, src_block_off, tokens, page_off,
                  R, total_pages, frag, raw_out, partial_out, error_flag, stream);
}

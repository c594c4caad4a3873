// Trigonometric key scorer on the 5th-generation tensor cores (tcgen05,
// sm_100a) with the fp32 accumulator in tensor memory (TMEM).
//
// Same contraction as the mma.sync scorer (kvc_score_tc.cuh), issued per unit
// (scoring layer, KV head, 128-token page) as M = 128 tokens x N = 16 columns
// x K = 16 tcgen05.mma steps accumulating into 16 TMEM columns.
//
// Roles of a CTA (one per SM, persistent over a contiguous range of units;
// units are dealt round-robin to the compute warpgroups):
//  * producer (one lane): streams each unit's key tile (128 tokens x
//    head_dim) from the paged cache with 4-D TMA box loads (128-byte swizzle)
//    into a ring of shared-memory stages, and bulk-copies the W matrix of the
//    unit's (request, layer, head) into one of two W buffers when it changes;
//  * compute warpgroups (kWg x 128 threads): thread t owns token t of the
//    page, which is TMEM lane t.  It reads its kr / ki row from the stage,
//    forms m = |(kr, ki)| split into 16-bit hi + lo, and stores kr | ki |
//    m_hi | m_lo into its warpgroup's TMEM columns (tcgen05.st): the A
//    operand of the rotary band.  After the MMAs it loads its 16 accumulator
//    columns (tcgen05.ld), adds the hi and lo halves per query head, and
//    writes the raw scores and the 32-token moments partials;
//  * MMA issuer (one lane): F/4 tcgen05.mma with A in TMEM, then P/16 with A
//    read from the stage through a shared-memory descriptor (the pass band
//    needs no arithmetic); B = W through a descriptor.  tcgen05.commit
//    arrives on the warpgroup's accumulator barrier (and on the stage's empty
//    barrier when the pass band was read from it).
// Every wait is bounded (KVC_DEV_TIMEOUT); a role that gives up stops, every
// thread meets at the final CTA barrier after copies and MMAs in flight have
// drained, and the allocating warp frees TMEM before the CTA exits.
//
// W layout (prepare_w_umma_kernel): per (request, layer, head) a K-major
// 16-row matrix of 16-bit values in the 128-byte-swizzled form the MMA
// descriptors read: K split into chunks of 64, each chunk 16 rows x 128 B
// (two 8-row groups of 1024 B), the 16-byte unit u of row n stored at
// position u ^ (n % 8) -- the pattern TMA writes for the key tiles.
#include <type_traits>

#include "kvc_score_tc.cuh"

namespace kvc {
namespace {

constexpr int kWg = 3;                        // compute warpgroups
constexpr int kProducerWarp = 4 * kWg;
constexpr int kMmaWarp = 4 * kWg + 1;
constexpr int kUmmaThreads = (4 * kWg + 2) * 32;
constexpr int kTmemCols = 512;                // all of TMEM: one CTA per SM
constexpr int kAccCols = 16;                  // N = 8 hi + 8 lo columns
constexpr int kSmemBudget = 220 * 1024;

struct UMeta {
  int p, h, lg, valid, wgen, skip;
  float scale;  // undoes the W scaling of the unit's (request, layer, head)
};

template <int F, int P>
struct UGeom {
  static constexpr int D = 2 * F + P;
  static constexpr int kBoxes = D / kBoxElems;
  static constexpr int kStageBytes = kBoxes * kBoxBytes;
  static constexpr int kWK = 4 * F + P;          // K extent of W
  static constexpr int kWBytes = kWK * 2 * 16;   // 16 rows of kWK 16-bit values
  static constexpr int kFit = (kSmemBudget - 2 * kWBytes) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  // TMEM columns of one warpgroup: A words (kr | ki | m_hi | m_lo, F/2 each)
  // then the accumulator, rounded to 32 columns
  static constexpr int kWgCols = (2 * F + kAccCols + 31) / 32 * 32;
  // barriers: full, empty [kStages]; aready, accfull [kWg]; wfull, wfree [2]; done
  static constexpr int kBars = 2 * kStages + 2 * kWg + 5;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + 2 * kWBytes + 8 * kBars +
                               (int)sizeof(UMeta) * (kStages + kWg) + 16;
  static_assert(D % kBoxElems == 0 && kWK % 64 == 0 && F % 32 == 0 && P % 16 == 0, "geometry");
  static_assert(kStages >= 2, "two stages at least");
  static_assert(kWg * kWgCols <= kTmemCols, "TMEM columns");
  static_assert(kSmem > 116 * 1024, "one CTA per SM: it holds every TMEM column");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

// ---------------------------------------------------------------------------
// tcgen05 / TMEM helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// arrives on `bar` once every tcgen05.mma this thread issued before has completed
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 8 consecutive 32-bit columns of this thread's lane (lane field of taddr =
// the warp's 32-lane slice)
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// load and wait in one statement, so no use of v can be scheduled before the wait
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void lds128(uint32_t addr, uint32_t* v) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(addr));
}

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzled layout: rows of 128 B, 8-row groups 1024 B apart.  `addr` is the
// first row of the 16-element K slice: a 1024-B aligned group base plus 32 B
// per K step inside the 128-byte span.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu)  // start address, 16-byte units
         | ((uint64_t)1 << 16)              // leading byte offset (not used by swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)    // stride byte offset: the next 8-row group
         | ((uint64_t)1 << 46)              // descriptor version of sm_100
         | ((uint64_t)2 << 61);             // 128-byte swizzle
}

// Instruction descriptor, kind::f16: f32 accumulator, A and B of the cache's
// 16-bit type, both K-major, N = kAccCols, M = 128.
constexpr uint32_t idesc_f16(bool fp16) {
  return (1u << 4) | ((fp16 ? 0u : 1u) << 7) | ((fp16 ? 0u : 1u) << 10) | ((uint32_t)(kAccCols >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}

// D (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// D (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// ---------------------------------------------------------------------------
// W in the swizzled K-major layout (one CTA per (layer, request, head))
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) prepare_w_umma_kernel(const __grid_constant__ FragArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  extern __shared__ float sm[];
  const int l = blockIdx.x, r = blockIdx.y, h = blockIdx.z;
  __shared__ float red[8];
  stage_w_inputs(a, sm, l, r, h);
  const float scale = w_scale(a, sm, l, h, red);
  const int KW = 4 * a.F + a.P;
  // this (request, layer, head)'s record: the swizzled matrix, then the inverse scale
  uint8_t* dst = reinterpret_cast<uint8_t*>(a.frag) + ((int64_t)(r * a.L + l) * a.kvh + h) * w_record_bytes(a.F, a.P);
  if (threadIdx.x == 0)
    *reinterpret_cast<uint4*>(dst + (int64_t)KW * 32) = make_uint4(__float_as_uint(1.f / scale), 0u, 0u, 0u);
  for (int i = threadIdx.x; i < 16 * (KW / 8); i += blockDim.x) {
    const int n = i & 15;      // row: n < 8 hi half of head n, else lo half of head n - 8
    const int k0 = (i >> 4) * 8;
    const int g = n & 7;
    uint32_t words[4] = {0u, 0u, 0u, 0u};
    for (int e = 0; e < 8; ++e) {
      bool lo_zero = false;
      const float v = g < a.G ? w_value(a, sm, l, h, g, k0 + e, lo_zero) * scale : 0.f;
      const uint16_t hi = to_half_bits(v, a.half_fp16);
      const uint16_t bits =
          n < 8 ? hi : lo_zero ? (uint16_t)0 : to_half_bits(v - from_half_bits(hi, a.half_fp16), a.half_fp16);
      words[e >> 1] |= (uint32_t)bits << (16 * (e & 1));
    }
    const int off = (k0 / 64) * 2048 + n * 128 + ((((k0 % 64) / 8) ^ (n & 7)) << 4);
    *reinterpret_cast<uint4*>(dst + off) = make_uint4(words[0], words[1], words[2], words[3]);
  }
}

// ---------------------------------------------------------------------------
// the scorer
// ---------------------------------------------------------------------------

template <int F, int P, bool FP16>
__global__ void __launch_bounds__(kUmmaThreads, 1) score_umma_kernel(const __grid_constant__ TcArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  using Gm = UGeom<F, P>;
  using E = std::conditional_t<FP16, Fp16, Bf16>;
  constexpr int S = Gm::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t stage0 = smem_u32(base);
  const uint32_t wbuf0 = stage0 + S * Gm::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + S * Gm::kStageBytes + 2 * Gm::kWBytes);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * S;
  const uint32_t aready0 = empty0 + 8 * S;    // A operand of the warpgroup's unit is in TMEM
  const uint32_t accfull0 = aready0 + 8 * kWg;  // the warpgroup's accumulator is complete
  const uint32_t wfull0 = accfull0 + 8 * kWg;
  const uint32_t wfree0 = wfull0 + 16;
  const uint32_t done = wfree0 + 16;
  UMeta* meta = reinterpret_cast<UMeta*>(bars + Gm::kBars);  // [S] per stage, from the producer
  UMeta* wmeta = meta + S;                                    // [kWg] per warpgroup, for the MMA issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wmeta + kWg);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, P > 0 ? 5 : 4);  // the 4 warps that read the stage (+ the MMA commit)
    }
    for (int w = 0; w < kWg; ++w) {
      mbar_init(aready0 + 8 * w, 128);
      mbar_init(accfull0 + 8 * w, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(wfull0 + 8 * b, 1);
      mbar_init(wfree0 + 8 * b, 1);
    }
    mbar_init(done, 1);
    mbar_init_fence();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int64_t per = (a.units + gridDim.x - 1) / gridDim.x;
  const int64_t u0 = (int64_t)blockIdx.x * per;
  const int64_t n = u0 < a.units ? min64(a.units, u0 + per) - u0 : 0;

  if (warp == kProducerWarp) {
    // ---------------- producer -------------------------------------------------
    if (lane == 0) {
      uint32_t it = 0;  // units published
      int r = 0, cur_key = -1, gen = -1, loaded = -1;
      float wscale = 1.f;
      for (int64_t u = u0; u < u0 + n; ++u) {
        const int p = (int)(u % a.total_pages);
        const int h = (int)((u / a.total_pages) % a.kvh);
        const int l = (int)(u / ((int64_t)a.total_pages * a.kvh));
        if (u == u0 || p == 0) r = request_of_page(a.page_off, a.R, p);
        while (__ldg(a.page_off + r + 1) <= p) ++r;  // units advance page by page
        const int pl = p - __ldg(a.page_off + r);
        const int64_t blk = __ldg(a.src_blocks + __ldg(a.src_block_off + r) + pl);
        const int lg = a.layer0 + l;
        const int s = it % S;
        if (!mbar_wait(empty0 + 8 * s, ((it / S) & 1) ^ 1, a.error_flag)) break;
        if (blk < 0 || blk >= a.num_blocks) {
          // the unit still takes its turn (no copy, no MMA), so every role counts the same units
          raise_flag(a.error_flag, KVC_DEV_BLOCK_RANGE);
          meta[s] = UMeta{p, h, lg, 0, gen, 1, 1.f};
          mbar_arrive(full0 + 8 * s);
          ++it;
          continue;
        }
        const int key = (r * a.L_total + lg) * a.kvh + h;
        const bool new_w = key != cur_key;
        if (new_w) {
          cur_key = key;
          ++gen;
          wscale = __ldg(reinterpret_cast<const float*>(a.frag + (int64_t)key * (Gm::kWBytes / 16 + 1) +
                                                        Gm::kWBytes / 16));
        }
        meta[s] = UMeta{p, h, lg, min(kBlock, __ldg(a.tokens + r) - pl * kBlock), gen, 0, wscale};
        mbar_expect_tx(full0 + 8 * s, Gm::kStageBytes);
#pragma unroll
        for (int b = 0; b < Gm::kBoxes; ++b)
          tma_load_4d(stage0 + s * Gm::kStageBytes + b * kBoxBytes, &a.maps[l], b * kBoxElems, h, 0, (int)blk,
                      full0 + 8 * s);
        ++it;
        if (new_w) {
          // buffer gen % 2 last held generation gen - 2: the MMA issuer releases it
          // when it moves past generation gen - 1
          const int wb = gen & 1;
          if (gen >= 2 && !mbar_wait(wfree0 + 8 * wb, ((gen >> 1) - 1) & 1, a.error_flag)) break;
          mbar_expect_tx(wfull0 + 8 * wb, Gm::kWBytes);
          bulk_load(wbuf0 + wb * Gm::kWBytes, a.frag + (int64_t)key * (Gm::kWBytes / 16 + 1), Gm::kWBytes,
                    wfull0 + 8 * wb);
          loaded = gen;
        }
      }
      // drain: every issued copy must have landed before the CTA may exit
      for (uint32_t k = 0; k < (uint32_t)S && k < it; ++k) {
        const uint32_t j = it - 1 - k;
        if (!mbar_wait(full0 + 8 * (j % S), (j / S) & 1, a.error_flag)) break;
      }
      for (int g = loaded; g >= 0 && g > loaded - 2; --g) mbar_wait(wfull0 + 8 * (g & 1), (g >> 1) & 1, a.error_flag);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer -----------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(FP16);
      int cur = -1;
      for (int64_t i = 0; i < n; ++i) {
        const int w = (int)(i % kWg);
        const int s = (int)(i % S);
        if (!mbar_wait(aready0 + 8 * w, (uint32_t)(i / kWg) & 1, a.error_flag)) break;
        tc_fence_after();
        const UMeta mu = wmeta[w];
        if (mu.skip) {
          mbar_arrive(accfull0 + 8 * w);
          if (P > 0) mbar_arrive(empty0 + 8 * s);
          continue;
        }
        if (mu.wgen != cur) {
          if (cur >= 0) tc_commit(wfree0 + 8 * (cur & 1));  // generation cur's buffer, once its MMAs are done
          if (!mbar_wait(wfull0 + 8 * (mu.wgen & 1), (mu.wgen >> 1) & 1, a.error_flag)) break;
          cur = mu.wgen;
        }
        // the pass band is read from the stage by the MMA itself: order it after the TMA bytes
        if (P > 0 && !mbar_wait(full0 + 8 * s, (uint32_t)(i / S) & 1, a.error_flag)) break;
        const uint32_t acol = tmem + w * Gm::kWgCols;
        const uint32_t d = acol + 2 * F;
        const uint32_t wb = wbuf0 + (cur & 1) * Gm::kWBytes;
#pragma unroll
        for (int j = 0; j < F / 4; ++j)
          mma_ts(d, acol + 8 * j, sw128_desc(wb + (j >> 2) * 2048 + (j & 3) * 32), idesc, j > 0 ? 1u : 0u);
        if constexpr (P > 0) {
          const uint32_t st = stage0 + s * Gm::kStageBytes;
#pragma unroll
          for (int j = 0; j < P / 16; ++j) {
            const int e = 2 * F + 16 * j;  // first key element of the K slice
            const int k = F / 4 + j;       // W K step
            mma_ss(d, sw128_desc(st + (e / kBoxElems) * kBoxBytes + (e % kBoxElems) * 2),
                   sw128_desc(wb + (k >> 2) * 2048 + (k & 3) * 32), idesc, 1u);
          }
        }
        tc_commit(accfull0 + 8 * w);
        if (P > 0) tc_commit(empty0 + 8 * s);
      }
      tc_commit(done);  // arrives once every MMA issued above has completed
      mbar_wait(done, 0, a.error_flag);
    }
    __syncwarp();
  } else {
    // ---------------- compute warpgroups ----------------------------------------
    // Per warpgroup: while the MMAs of unit k run, the key rows of unit k+1
    // are read into registers (releasing the stage) and unit k-1's scores are
    // written; once unit k's accumulator is read, unit k+1's A operand is
    // formed into the same TMEM columns and handed to the issuer.
    const int wg = warp >> 2, q = warp & 3;
    const int t = threadIdx.x & 127;  // token of the page = TMEM lane
    const uint32_t acol = tmem + ((uint32_t)(32 * q) << 16) + wg * Gm::kWgCols;
    const uint32_t row_off = t * 128;
    const int sw = t & 7;
    const int heads = a.kvh * a.G;
    uint32_t kr[F / 2], ki[F / 2];

    // unit i's kr / ki rows into registers
    auto load = [&](int64_t i, UMeta& mu) -> bool {
      const int s = (int)(i % S);
      // waits are voted warp-wide, so a timed-out warp leaves as a whole
      if (!__all_sync(0xffffffffu, mbar_wait(full0 + 8 * s, (uint32_t)(i / S) & 1, a.error_flag))) return false;
      mu = meta[s];
      if (!mu.skip) {
        const uint32_t row = stage0 + s * Gm::kStageBytes + row_off;
#pragma unroll
        for (int c = 0; c < F / 8; ++c) {
          const int er = 8 * c, ei = F + er;
          lds128(row + (er / kBoxElems) * kBoxBytes + ((((er % kBoxElems) / 8) ^ sw) << 4), kr + 4 * c);
          lds128(row + (ei / kBoxElems) * kBoxBytes + ((((ei % kBoxElems) / 8) ^ sw) << 4), ki + 4 * c);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);  // this warp is done reading the stage
      return true;
    };
    // A operand kr | ki | m_hi | m_lo (m = |(kr, ki)| split into hi + lo) into
    // this warpgroup's TMEM columns, then hand the unit to the MMA issuer
    auto form_a = [&](const UMeta& mu) {
      if (!mu.skip) {
#pragma unroll
        for (int grp = 0; grp < F / 16; ++grp) {  // 16 frequencies (8 columns per band) at a time
          uint32_t mh[8], ml[8];
          modulus_split<E>(kr + 8 * grp, ki + 8 * grp, mh, ml);
          modulus_split<E>(kr + 8 * grp + 4, ki + 8 * grp + 4, mh + 4, ml + 4);
          tmem_st8(acol + 8 * grp, kr + 8 * grp);
          tmem_st8(acol + F / 2 + 8 * grp, ki + 8 * grp);
          tmem_st8(acol + F + 8 * grp, mh);
          tmem_st8(acol + 3 * F / 2 + 8 * grp, ml);
        }
      }
      if (t == 0) wmeta[wg] = mu;
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(aready0 + 8 * wg);
    };
    // raw scores, and per query head the 32-token moments (sum, sum of squared
    // deviations from the slice mean) of this warp's slice
    auto epilogue = [&](const UMeta& mu, const float* yv) {
      const bool tv = t < mu.valid;
      const int nq = max(0, min(32, mu.valid - 32 * q));
      float* out = a.raw + (((int64_t)mu.lg * a.total_pages + mu.p) * heads + mu.h * a.G) * kBlock + t;
      // x[g] = sum terms, x[8 + g] = squares about c[g] (token 32q's score: a
      // value inside the data, so the correction below cancels nothing big)
      float x[16], c[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const float y = yv[g];
        c[g] = 0.f;
        if (g < a.G) {
          if (tv) out[g * kBlock] = y;
          c[g] = __shfl_sync(0xffffffffu, y, 0);
        }
        const float d = y - c[g];
        x[g] = tv ? y : 0.f;
        x[8 + g] = tv ? d * d : 0.f;
      }
      // transpose-reduce: after the step of distance d every lane keeps half of
      // its values (the half its lane bit selects) summed with its partner's;
      // lane l ends with value (l >> 1) & 15 summed over the 32 lanes
#pragma unroll
      for (int m = 8; m >= 1; m >>= 1) {
        const int d = 2 * m;
        const bool up = (lane & d) != 0;
#pragma unroll
        for (int i = 0; i < m; ++i) {
          const float send = up ? x[i] : x[i + m];
          const float keep = up ? x[i + m] : x[i];
          x[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
        }
      }
      x[0] += __shfl_xor_sync(0xffffffffu, x[0], 1);
      // lanes 2g hold head g's sum, lanes 16 + 2g its squares about c[g]
      const float sq = __shfl_xor_sync(0xffffffffu, x[0], 16);
      const int g = lane >> 1;
      if (lane < 16 && (lane & 1) == 0 && g < a.G) {
        float cg = c[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) cg = g == j ? c[j] : cg;
        float m2 = 0.f;
        if (nq > 0) {
          const float e = x[0] - (float)nq * cg;  // n * (mean - c)
          m2 = fmaxf(0.f, sq - e * e * __frcp_rn((float)nq));
        }
        float2* part = reinterpret_cast<float2*>(a.partial) +
                       (((int64_t)mu.lg * a.total_pages + mu.p) * kTcQuarters + q) * heads + mu.h * a.G;
        part[g] = make_float2(x[0], m2);
      }
    };

    UMeta cur{}, nxt{};
    if (wg < n && load(wg, cur)) {
      form_a(cur);
      for (int64_t k = 0;; ++k) {
        const int64_t inext = wg + (k + 1) * kWg;
        const bool more = inext < n;
        if (more && !load(inext, nxt)) break;
        if (!__all_sync(0xffffffffu, mbar_wait(accfull0 + 8 * wg, (uint32_t)k & 1, a.error_flag))) break;
        tc_fence_after();
        float y[8];  // unit k's scores: hi-column plus lo-column products per query head
        if (!cur.skip) {
          uint32_t v[16];
          tmem_ld16(acol + 2 * F, v);
#pragma unroll
          for (int g = 0; g < 8; ++g) y[g] = (__uint_as_float(v[g]) + __uint_as_float(v[8 + g])) * cur.scale;
        }
        if (more) form_a(nxt);  // the MMAs of unit k have read A; its accumulator is in y
        if (!cur.skip) epilogue(cur, y);
        if (!more) break;
        cur = nxt;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int F, int P, bool FP16>
int launch_t(const TcArgs& a, cudaStream_t st) {
  using Gm = UGeom<F, P>;
  if (a.units == 0) return KVC_OK;
  static bool configured[64] = {};  // per device: the shared-memory opt-in is a per-context attribute
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KVC_ECUDA;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(score_umma_kernel<F, P, FP16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Gm::kSmem) != cudaSuccess)
      return KVC_ECUDA;
    configured[dev] = true;
  }
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(sm_count(), a.units));
  launch_dep(score_umma_kernel<F, P, FP16>, dim3(grid), dim3(kUmmaThreads), (size_t)Gm::kSmem, st, a);
  return launch_status();
}

template <bool FP16>
int dispatch(const TcArgs& a, int F, int P, cudaStream_t st) {
  if (F == 64 && P == 0) return launch_t<64, 0, FP16>(a, st);
  if (F == 32 && P == 0) return launch_t<32, 0, FP16>(a, st);
  if (F == 32 && P == 192) return launch_t<32, 192, FP16>(a, st);
  if (F == 32 && P == 64) return launch_t<32, 64, FP16>(a, st);
  if (F == 64 && P == 128) return launch_t<64, 128, FP16>(a, st);
  return KVC_EUNSUPPORTED;
}

}  // namespace

bool umma_geometry(int F, int P) {
  return (F == 64 && P == 0) || (F == 32 && P == 0) || (F == 32 && P == 192) || (F == 32 && P == 64) ||
         (F == 64 && P == 128);
}

int prepare_w_umma(const FragArgs& a, cudaStream_t st) {
  const size_t smem = w_stage_floats(a.n_off, a.F, a.G) * sizeof(float);
  launch_dep(prepare_w_umma_kernel, dim3(a.L, a.R, a.kvh), dim3(256), smem, st, a);
  return launch_status();
}

int launch_umma(const TcArgs& a, int F, int P, bool fp16, cudaStream_t st) {
  return fp16 ? dispatch<true>(a, F, P, st) : dispatch<false>(a, F, P, st);
}

}  // namespace kvc

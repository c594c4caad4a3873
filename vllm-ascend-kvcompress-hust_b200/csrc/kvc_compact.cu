// Paged K/V compaction, slot gather/scatter and decode position shift (sm_100a).
//
// Compaction moves N_layers * 2 * R * budget token rows (row = all local KV
// heads of one token, contiguous in the [blocks][128][kvh][D] layout).  Each
// warp owns a tile of 32 consecutive output rows: lane i resolves row i's
// source/destination addresses (keep index -> source block -> address, with
// range checks) so the dependent index loads of 32 rows overlap; the warp then
// streams the rows with 16-byte vectors (narrower when the caller's strides or
// bases are not 16-byte aligned), two rows in flight per pass.  Rows under
// 2 KB (few local heads under tensor parallelism) are copied as one flat
// (row, vector) range per tile so each lane still has eight vectors in flight.
#include "kvc_async.cuh"

namespace kvc {

constexpr int kMaxCompactLayers = 512;
constexpr int kCopyThreads = 256;

struct CompactArgs {
  const void* k_layers[kMaxCompactLayers];
  const void* v_layers[kMaxCompactLayers];
  int64_t block_stride;  // bytes
  int64_t num_blocks;
  int64_t row_bytes;
  const int64_t* src_blocks;
  const int64_t* src_block_off;
  const int64_t* dst_blocks;
  const int64_t* dst_block_off;
  const int64_t* keep;
  const int32_t* tokens;
  int32_t* error_flag;
  int N, R, budget, tile_rows;
  int nvec_shift;  // log2(row_bytes / vector width) when a power of two, else -1
};

template <int VEC>
struct Vec;
struct alignas(32) U32x8 {
  uint32_t w[8];
};
template <> struct Vec<32> { using T = U32x8; };
template <> struct Vec<16> { using T = uint4; };
template <> struct Vec<8> { using T = uint2; };
template <> struct Vec<4> { using T = uint32_t; };
template <> struct Vec<2> { using T = uint16_t; };

template <int VEC>
__device__ __forceinline__ typename Vec<VEC>::T load_nc(const void* p) {
  using T = typename Vec<VEC>::T;
  if constexpr (VEC == 32) {  // one 256-bit load (sm_100)
    T r;
    asm("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3]), "=r"(r.w[4]), "=r"(r.w[5]), "=r"(r.w[6]),
          "=r"(r.w[7])
        : "l"(p));
    return r;
  } else if constexpr (VEC == 16) {
    return ldg_stream16(p);
  } else {
    return __ldg(reinterpret_cast<const T*>(p));
  }
}

template <int VEC>
__device__ __forceinline__ void store_vec(void* p, const typename Vec<VEC>::T& x) {
  using T = typename Vec<VEC>::T;
  if constexpr (VEC == 32) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(x.w[0]), "r"(x.w[1]),
                 "r"(x.w[2]), "r"(x.w[3]), "r"(x.w[4]), "r"(x.w[5]), "r"(x.w[6]), "r"(x.w[7])
                 : "memory");
  } else {
    *reinterpret_cast<T*>(p) = x;
  }
}

// Resolve (src, dst) byte addresses of output row q; nullptr on a range fault.
__device__ __forceinline__ void resolve_row(const CompactArgs& a, int64_t q, const char*& src, char*& dst) {
  src = nullptr;
  dst = nullptr;
  const int64_t j = q % a.budget;
  int64_t t = q / a.budget;
  const int r = (int)(t % a.R);
  t /= a.R;
  const int kv = (int)(t & 1);
  const int layer = (int)(t >> 1);
  const int64_t idx = __ldg(a.keep + (int64_t)r * a.budget + j);
  if (idx < 0 || idx >= __ldg(a.tokens + r)) {
    raise_flag(a.error_flag, KVC_DEV_TOKEN_RANGE);
    return;
  }
  const int64_t sb = __ldg(a.src_blocks + __ldg(a.src_block_off + r) + (idx >> 7));
  const int64_t db = __ldg(a.dst_blocks + __ldg(a.dst_block_off + r) + (j >> 7));
  if (sb < 0 || sb >= a.num_blocks || db < 0 || db >= a.num_blocks) {
    raise_flag(a.error_flag, KVC_DEV_BLOCK_RANGE);
    return;
  }
  const char* base_s = reinterpret_cast<const char*>(kv ? a.v_layers[layer] : a.k_layers[layer]);
  char* base_d = const_cast<char*>(base_s);
  src = base_s + sb * a.block_stride + (idx & 127) * a.row_bytes;
  dst = base_d + db * a.block_stride + (j & 127) * a.row_bytes;
}

// resolve_row in three stages, so that a warp copying narrow rows can issue
// the next tile's dependent index loads between its copy passes: begin loads
// the keep index and the request's offsets, middle the two block ids, end
// checks the ranges and forms the addresses (same checks and flags).
struct RowFetch {
  int64_t q;  // -1: no row
  int64_t idx, soff, doff, sb, db;
  int32_t ntok;
};

__device__ __forceinline__ void fetch_begin(const CompactArgs& a, int64_t q, RowFetch& f) {
  f.q = q;
  if (q < 0) return;
  const int64_t j = q % a.budget;
  const int r = (int)((q / a.budget) % a.R);
  f.idx = __ldg(a.keep + (int64_t)r * a.budget + j);
  f.ntok = __ldg(a.tokens + r);
  f.soff = __ldg(a.src_block_off + r);
  f.doff = __ldg(a.dst_block_off + r);
}

__device__ __forceinline__ void fetch_middle(const CompactArgs& a, RowFetch& f) {
  if (f.q < 0) return;
  const int64_t j = f.q % a.budget;
  f.sb = (f.idx >= 0 && f.idx < f.ntok) ? __ldg(a.src_blocks + f.soff + (f.idx >> 7)) : -1;
  f.db = __ldg(a.dst_blocks + f.doff + (j >> 7));
}

__device__ __forceinline__ void fetch_end(const CompactArgs& a, const RowFetch& f, const char*& src, char*& dst) {
  src = nullptr;
  dst = nullptr;
  if (f.q < 0) return;
  if (f.idx < 0 || f.idx >= f.ntok) {
    raise_flag(a.error_flag, KVC_DEV_TOKEN_RANGE);
    return;
  }
  if (f.sb < 0 || f.sb >= a.num_blocks || f.db < 0 || f.db >= a.num_blocks) {
    raise_flag(a.error_flag, KVC_DEV_BLOCK_RANGE);
    return;
  }
  const int64_t j = f.q % a.budget;
  const int64_t t = f.q / a.budget / a.R;
  const int kv = (int)(t & 1);
  const int layer = (int)(t >> 1);
  const char* base = reinterpret_cast<const char*>(kv ? a.v_layers[layer] : a.k_layers[layer]);
  src = base + f.sb * a.block_stride + (f.idx & 127) * a.row_bytes;
  dst = const_cast<char*>(base) + f.db * a.block_stride + (j & 127) * a.row_bytes;
}

template <int VEC, bool SMALL>
__global__ void __launch_bounds__(kCopyThreads, SMALL ? 2 : 4) compact_kernel(const __grid_constant__ CompactArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  using T = typename Vec<VEC>::T;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)a.N * 2 * a.R * a.budget;
  const int tr = a.tile_rows;  // rows per warp tile (<= 32; fewer for small problems)
  const int64_t tiles = (rows + tr - 1) / tr;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nvec = (int)(a.row_bytes / VEC);
  const char* next_src = nullptr;
  char* next_dst = nullptr;
  if constexpr (SMALL) {  // the first tile's rows; later tiles are resolved one tile ahead
    RowFetch f;
    const int64_t q = warp0 * tr + lane;
    fetch_begin(a, (warp0 < tiles && lane < tr && q < rows) ? q : -1, f);
    fetch_middle(a, f);
    fetch_end(a, f, next_src, next_dst);
  }
  for (int64_t tile = warp0; tile < tiles; tile += nwarps) {
    const int64_t q = tile * tr + lane;
    const char* my_src = nullptr;
    char* my_dst = nullptr;
    if constexpr (SMALL) {
      my_src = next_src;
      my_dst = next_dst;
    } else {
      if (lane < tr && q < rows) resolve_row(a, q, my_src, my_dst);
    }
    const int nrows = (int)min64(tr, rows - tile * tr);
    if constexpr (SMALL) {
      // rows narrower than 2 KB: spread the tile's (row, vector) pairs over the
      // lanes so that every lane keeps kSmallU vectors in flight; the next
      // tile's index loads run between the copy passes
      RowFetch nf;
      const int64_t nq = (tile + nwarps) * tr + lane;
      fetch_begin(a, (tile + nwarps < tiles && lane < tr && nq < rows) ? nq : -1, nf);
      constexpr int kSmallU = VEC == 32 ? 4 : 8;  // 128 (256) bytes in flight per lane
      const int total = nrows * nvec;
      bool middle_done = false;
      for (int e0 = 0; e0 < total; e0 += 32 * kSmallU) {
        if (e0 > 0 && !middle_done) {
          fetch_middle(a, nf);
          middle_done = true;
        }
        T x[kSmallU];
        char* dd[kSmallU];
#pragma unroll
        for (int u = 0; u < kSmallU; ++u) {
          const int e = e0 + u * 32 + lane;
          const int row = min(a.nvec_shift >= 0 ? e >> a.nvec_shift : e / nvec, nrows - 1);
          const char* s = (const char*)__shfl_sync(0xffffffffu, (unsigned long long)my_src, row);
          char* d = (char*)__shfl_sync(0xffffffffu, (unsigned long long)my_dst, row);
          dd[u] = nullptr;
          if (e < total && s) {
            const int64_t off = (int64_t)(e - row * nvec) * VEC;
            x[u] = load_nc<VEC>(s + off);
            dd[u] = d + off;
          }
        }
#pragma unroll
        for (int u = 0; u < kSmallU; ++u)
          if (dd[u]) store_vec<VEC>(dd[u], x[u]);
      }
      if (!middle_done) fetch_middle(a, nf);
      fetch_end(a, nf, next_src, next_dst);
    } else {
    constexpr int kU = VEC == 32 ? 2 : 4;  // vectors per lane per row in one pass
    for (int k = 0; k < nrows; k += 2) {
      const char* s0 = (const char*)__shfl_sync(0xffffffffu, (unsigned long long)my_src, k);
      char* d0 = (char*)__shfl_sync(0xffffffffu, (unsigned long long)my_dst, k);
      const int k1 = min(k + 1, nrows - 1);
      const char* s1 = (const char*)__shfl_sync(0xffffffffu, (unsigned long long)my_src, k1);
      char* d1 = (char*)__shfl_sync(0xffffffffu, (unsigned long long)my_dst, k1);
      if (k1 == k) { s1 = nullptr; d1 = nullptr; }
      for (int v0 = 0; v0 < nvec; v0 += 32 * kU) {
        T x0[kU], x1[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < nvec) {
            if (s0) x0[u] = load_nc<VEC>(s0 + (int64_t)v * VEC);
            if (s1) x1[u] = load_nc<VEC>(s1 + (int64_t)v * VEC);
          }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < nvec) {
            if (s0) store_vec<VEC>(d0 + (int64_t)v * VEC, x0[u]);
            if (s1) store_vec<VEC>(d1 + (int64_t)v * VEC, x1[u]);
          }
        }
      }
    }
    }
  }
}

// Bulk-copy variant (16-byte aligned rows up to kBulkWarpBytes / 2): the TMA
// engine moves whole rows.  One CTA per SM, kBulkWarps independent warps, each
// owning kBulkWarpBytes of shared memory split into two row sets.  Per group of
// up to 32 rows (one per lane): each lane bulk-loads its row into its slot of
// the current set (completion counted on the set's mbarrier), the warp waits
// for the set, then each lane bulk-stores its slot to the destination row and
// commits a bulk group.  The next group uses the other set, so its loads fly
// while the previous group's stores drain; a slot is reloaded only after the
// lane's store from it two groups earlier has finished reading it.
constexpr int kBulkWarps = 8;
constexpr int kBulkWarpBytes = 24 * 1024;
constexpr int kBulkSmem = kBulkWarps * kBulkWarpBytes;

__global__ void __launch_bounds__(kBulkWarps * 32, 1) compact_bulk_kernel(const __grid_constant__ CompactArgs a) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t bulk_sm[];
  __shared__ __align__(8) uint64_t bars[kBulkWarps][2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rb = (uint32_t)a.row_bytes;
  const int gs = min(32, (int)(kBulkWarpBytes / rb) / 2);  // rows per group (host: >= 1)
  const uint32_t buf = smem_u32(bulk_sm + warp * kBulkWarpBytes);
  const uint32_t bar0 = smem_u32(&bars[warp][0]);
  if (lane == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    mbar_init_fence();
  }
  __syncwarp();
  const int64_t rows = (int64_t)a.N * 2 * a.R * a.budget;
  const int tr = a.tile_rows;
  const int64_t tiles = (rows + tr - 1) / tr;
  const int64_t nwarps = (int64_t)gridDim.x * kBulkWarps;
  uint32_t parity = 0;  // bit s: phase parity of set s's barrier
  int grp = 0;
  bool ok = true;
  for (int64_t tile = (int64_t)blockIdx.x * kBulkWarps + warp; ok && tile < tiles; tile += nwarps) {
    const int64_t q = tile * tr + lane;
    const char* my_src = nullptr;
    char* my_dst = nullptr;
    if (lane < tr && q < rows) resolve_row(a, q, my_src, my_dst);
    const int nrows = (int)min64(tr, rows - tile * tr);
    for (int k0 = 0; ok && k0 < nrows; k0 += gs, ++grp) {
      const int set = grp & 1;
      const int from = min(k0 + lane, 31);
      const char* s = (const char*)__shfl_sync(0xffffffffu, (unsigned long long)my_src, from);
      char* d = (char*)__shfl_sync(0xffffffffu, (unsigned long long)my_dst, from);
      const bool mine = lane < min(gs, nrows - k0) && s != nullptr;
      const unsigned mask = __ballot_sync(0xffffffffu, mine);
      bulk_wait_read<1>();  // this lane's store from this set (two groups ago) has read its slot
      if (mask) {
        const uint32_t bar = bar0 + 8 * set;
        const uint32_t slot = buf + (uint32_t)(set * gs + lane) * rb;
        if (lane == 0) mbar_expect_tx(bar, (uint32_t)__popc(mask) * rb);
        __syncwarp();
        if (mine) bulk_load(slot, s, rb, bar);
        // one verdict for the whole warp: a lane that saw the phase complete and a
        // lane whose bound expired must leave (or go on) together, since the
        // next group's shuffles and ballot name every lane
        ok = __all_sync(0xffffffffu, mbar_wait(bar, (parity >> set) & 1u, a.error_flag));
        if (!ok) mbar_wait(bar, (parity >> set) & 1u, nullptr);  // let loads in flight land before exiting
        parity ^= 1u << set;
        if (ok && mine) bulk_store(d, slot, rb);
      }
      bulk_commit();  // one group per lane per round, empty or not, so wait_read<1> means "two rounds ago"
    }
  }
  bulk_wait_all();
}

// Commit staging of request r: its destination row (one entry per scheduler
// page of `bpp` kernel blocks: the page id is its first block / bpp; entries
// past the request's pages are -1) and its position offset semantic - budget.
__global__ void stage_commit_kernel(const int64_t* __restrict__ dst_blocks, const int64_t* __restrict__ dst_block_off,
                                    int R, int bpp, int64_t* staged_rows, int stride, int64_t* staged_offsets,
                                    const int64_t* __restrict__ semantic, int budget) {
  pdl_wait();  // the preceding kernel of the step has finished (see kvc_common.cuh)
  pdl_trigger();
  const int r = blockIdx.x;
  const int64_t b0 = dst_block_off[r], b1 = dst_block_off[r + 1];
  if (staged_rows)
    for (int64_t i = threadIdx.x; i < stride; i += blockDim.x)
      staged_rows[(int64_t)r * stride + i] = (b0 + i * bpp < b1) ? dst_blocks[b0 + i * bpp] / bpp : -1;
  if (staged_offsets && semantic && threadIdx.x == 0) staged_offsets[r] = semantic[r] - budget;
}

// ---- slot gather / scatter (workspace path of the cache API) -------------

template <int VEC, bool GATHER>
__global__ void __launch_bounds__(kCopyThreads) slots_kernel(const char* cache_in, char* cache_out,
                                                             int64_t block_stride, int block_size,
                                                             int64_t num_blocks, int64_t row_bytes,
                                                             const int64_t* __restrict__ slots, int64_t n,
                                                             const char* ws_in, char* ws_out, int32_t* flag) {
  using T = typename Vec<VEC>::T;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nvec = (int)(row_bytes / VEC);
  for (int64_t i = warp0; i < n; i += nwarps) {
    const int64_t slot = __ldg(slots + i);
    const int64_t blk = slot / block_size;
    if (slot < 0 || blk >= num_blocks) {
      if (lane == 0) raise_flag(flag, KVC_DEV_BLOCK_RANGE);
      continue;
    }
    const int64_t off = blk * block_stride + (slot % block_size) * row_bytes;
    for (int v = lane; v < nvec; v += 32) {
      if (GATHER)
        *reinterpret_cast<T*>(ws_out + i * row_bytes + (int64_t)v * VEC) =
            *reinterpret_cast<const T*>(cache_in + off + (int64_t)v * VEC);
      else
        *reinterpret_cast<T*>(cache_out + off + (int64_t)v * VEC) =
            *reinterpret_cast<const T*>(ws_in + i * row_bytes + (int64_t)v * VEC);
    }
  }
}

template <typename I>
__global__ void shift_positions_kernel(const int64_t* __restrict__ pos, const I* __restrict__ req,
                                       const int64_t* __restrict__ offsets, int64_t num_offsets, int64_t n,
                                       int64_t* out, int32_t* flag) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t r = (int64_t)req[i];
  if (r < 0 || r >= num_offsets) {
    raise_flag(flag, KVC_DEV_INDEX_RANGE);
    out[i] = pos[i];
    return;
  }
  out[i] = pos[i] - offsets[r];
}

inline int vec_width(uintptr_t bits) {
  if (bits % 16 == 0) return 16;
  if (bits % 8 == 0) return 8;
  if (bits % 4 == 0) return 4;
  if (bits % 2 == 0) return 2;
  return 0;
}

inline unsigned copy_grid(int64_t work_warps, int blocks_per_sm = 2048 / kCopyThreads) {
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm;
  const int64_t want = (work_warps * 32 + kCopyThreads - 1) / kCopyThreads;
  return (unsigned)std::max<int64_t>(1, std::min(cap, want));
}

// Resident CTAs per SM of one compaction variant (register-limited), so the
// grid-stride loop runs as a single wave.
template <int VEC, bool SMALL>
int compact_blocks_per_sm() {
  static int n = 0;
  if (n == 0) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, compact_kernel<VEC, SMALL>, kCopyThreads, 0) != cudaSuccess ||
        b <= 0)
      b = 2048 / kCopyThreads;
    n = b;
  }
  return n;
}

// One-time opt-in to the bulk kernel's shared memory (per device, first call before any capture).
bool bulk_ready() {
  static int state[64] = {0};  // 0 unknown, 1 ready, -1 unavailable
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (state[dev] == 0)
    state[dev] = cudaFuncSetAttribute(compact_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmem) ==
                         cudaSuccess
                     ? 1
                     : -1;
  if (state[dev] < 0) cudaGetLastError();
  return state[dev] > 0;
}

template <int VEC, bool SMALL>
void launch_compact(const CompactArgs& a, int64_t tiles, cudaStream_t st) {
  launch_dep(compact_kernel<VEC, SMALL>, dim3(copy_grid(tiles, compact_blocks_per_sm<VEC, SMALL>())),
             dim3(kCopyThreads), 0, st, a);
}

}  // namespace kvc

using namespace kvc;

extern "C" int kvc_compact(const void* const* k_layers, const void* const* v_layers, int N,
                           int64_t block_stride_bytes, int64_t num_blocks, int64_t row_bytes,
                           const int64_t* src_blocks, const int64_t* src_block_off, const int64_t* dst_blocks,
                           const int64_t* dst_block_off, const int64_t* keep, const int32_t* tokens, int R,
                           int budget, int64_t* staged_rows, int staged_row_stride, int64_t* staged_offsets,
                           const int64_t* semantic, int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(k_layers && v_layers && src_blocks && src_block_off && dst_blocks && dst_block_off && keep && tokens,
                KVC_ENULL);
  KVC_CHECK_ARG(N > 0 && R >= 0 && budget > 0 && row_bytes > 0 && num_blocks > 0, KVC_EINVAL);
  KVC_CHECK_ARG(block_stride_bytes >= (int64_t)kBlock * row_bytes, KVC_EINVAL);
  KVC_CHECK_ARG(staged_rows == nullptr || staged_row_stride > 0, KVC_EINVAL);
  if (R == 0) return KVC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  uintptr_t bits = (uintptr_t)block_stride_bytes | (uintptr_t)row_bytes;
  for (int i = 0; i < N; ++i) {
    KVC_CHECK_ARG(k_layers[i] && v_layers[i], KVC_ENULL);
    bits |= (uintptr_t)k_layers[i] | (uintptr_t)v_layers[i];
  }
  // 32-byte vectors (256-bit loads/stores) when every base, stride and row allows them
  const int vec = bits % 32 == 0 ? 32 : vec_width(bits);
  KVC_CHECK_ARG(vec > 0, KVC_EALIGN);
  for (int l0 = 0; l0 < N; l0 += kMaxCompactLayers) {
    CompactArgs a{};
    a.N = std::min(kMaxCompactLayers, N - l0);
    for (int i = 0; i < a.N; ++i) {
      a.k_layers[i] = k_layers[l0 + i];
      a.v_layers[i] = v_layers[l0 + i];
    }
    a.block_stride = block_stride_bytes;
    a.num_blocks = num_blocks;
    a.row_bytes = row_bytes;
    a.src_blocks = src_blocks;
    a.src_block_off = src_block_off;
    a.dst_blocks = dst_blocks;
    a.dst_block_off = dst_block_off;
    a.keep = keep;
    a.tokens = tokens;
    a.error_flag = error_flag;
    a.R = R;
    a.budget = budget;
    const int64_t rows = (int64_t)a.N * 2 * R * budget;
    // bulk copies pay off for rows of 1 KB and more (per-copy overhead dominates below)
    const bool bulk = vec >= 16 && row_bytes % 16 == 0 && row_bytes >= 1024 && row_bytes <= kBulkWarpBytes / 2 &&
                      bulk_ready();
    // enough warps to fill the GPU: shrink the per-warp tile when rows are few,
    // but give every warp of the chosen kernel all its rows in one tile (a warp
    // resolves and copies a tile's rows together; tiles run one after another)
    const int64_t warps = (int64_t)sm_count() * (bulk ? kBulkWarps : 2048 / 32);
    a.tile_rows = (int)std::max<int64_t>(1, std::min<int64_t>(32, bulk ? (rows + warps - 1) / warps : rows / warps));
    const int64_t nvec = row_bytes / vec;
    a.nvec_shift = (nvec & (nvec - 1)) == 0 ? __builtin_ctzll((unsigned long long)nvec) : -1;
    const int64_t tiles = (rows + a.tile_rows - 1) / a.tile_rows;
    if (bulk) {
      const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(sm_count(), (tiles + kBulkWarps - 1) / kBulkWarps));
      launch_dep(compact_bulk_kernel, dim3(grid), dim3(kBulkWarps * 32), kBulkSmem, st, a);
    } else if (row_bytes < 2048) {
      switch (vec) {
        case 32: launch_compact<32, true>(a, tiles, st); break;
        case 16: launch_compact<16, true>(a, tiles, st); break;
        case 8: launch_compact<8, true>(a, tiles, st); break;
        case 4: launch_compact<4, true>(a, tiles, st); break;
        default: launch_compact<2, true>(a, tiles, st); break;
      }
    } else {
      switch (vec) {
        case 32: launch_compact<32, false>(a, tiles, st); break;
        case 16: launch_compact<16, false>(a, tiles, st); break;
        case 8: launch_compact<8, false>(a, tiles, st); break;
        case 4: launch_compact<4, false>(a, tiles, st); break;
        default: launch_compact<2, false>(a, tiles, st); break;
      }
    }
    const int rc = launch_status();
    if (rc != KVC_OK) return rc;
  }
  if (staged_rows || (staged_offsets && semantic)) {
    launch_dep(stage_commit_kernel, dim3(R), dim3(128), 0, st, dst_blocks, dst_block_off, R, 1, staged_rows,
               staged_row_stride, staged_offsets, semantic, budget);
    return launch_status();
  }
  return KVC_OK;
}

extern "C" int kvc_stage_commit(const int64_t* dst_blocks, const int64_t* dst_block_off, int num_requests,
                                int blocks_per_page, int64_t* staged_rows, int staged_row_stride,
                                int64_t* staged_offsets, const int64_t* semantic, int budget, void* stream) {
  KVC_CHECK_ARG(dst_blocks && dst_block_off, KVC_ENULL);
  KVC_CHECK_ARG(staged_offsets == nullptr || semantic != nullptr, KVC_ENULL);
  KVC_CHECK_ARG(num_requests >= 0 && blocks_per_page >= 1 && budget > 0, KVC_EINVAL);
  KVC_CHECK_ARG(staged_rows == nullptr || staged_row_stride > 0, KVC_EINVAL);
  if (num_requests == 0 || (!staged_rows && !staged_offsets)) return KVC_OK;
  launch_dep(stage_commit_kernel, dim3(num_requests), dim3(128), 0, (cudaStream_t)stream, dst_blocks, dst_block_off,
             num_requests, blocks_per_page, staged_rows, staged_row_stride, staged_offsets, semantic, budget);
  return launch_status();
}

template <bool GATHER>
static int slots_launch(const void* cache_in, void* cache_out, int64_t block_stride_bytes, int block_size,
                        int64_t num_blocks, int64_t row_bytes, const int64_t* slots, int64_t n, const void* ws_in,
                        void* ws_out, int32_t* flag, void* stream) {
  KVC_CHECK_ARG(slots && (GATHER ? (cache_in && ws_out) : (cache_out && ws_in)), KVC_ENULL);
  KVC_CHECK_ARG(block_size > 0 && num_blocks > 0 && row_bytes > 0 && n >= 0, KVC_EINVAL);
  KVC_CHECK_ARG(block_stride_bytes >= (int64_t)block_size * row_bytes, KVC_EINVAL);
  if (n == 0) return KVC_OK;
  const uintptr_t bits = (uintptr_t)block_stride_bytes | (uintptr_t)row_bytes |
                         (uintptr_t)(GATHER ? cache_in : cache_out) | (uintptr_t)(GATHER ? ws_out : ws_in);
  const int vec = vec_width(bits);
  KVC_CHECK_ARG(vec > 0, KVC_EALIGN);
  const unsigned grid = copy_grid(n);
  cudaStream_t st = (cudaStream_t)stream;
  const char* ci = (const char*)cache_in;
  char* co = (char*)cache_out;
  const char* wi = (const char*)ws_in;
  char* wo = (char*)ws_out;
  switch (vec) {
    case 16: slots_kernel<16, GATHER><<<grid, kCopyThreads, 0, st>>>(ci, co, block_stride_bytes, block_size, num_blocks, row_bytes, slots, n, wi, wo, flag); break;
    case 8: slots_kernel<8, GATHER><<<grid, kCopyThreads, 0, st>>>(ci, co, block_stride_bytes, block_size, num_blocks, row_bytes, slots, n, wi, wo, flag); break;
    case 4: slots_kernel<4, GATHER><<<grid, kCopyThreads, 0, st>>>(ci, co, block_stride_bytes, block_size, num_blocks, row_bytes, slots, n, wi, wo, flag); break;
    default: slots_kernel<2, GATHER><<<grid, kCopyThreads, 0, st>>>(ci, co, block_stride_bytes, block_size, num_blocks, row_bytes, slots, n, wi, wo, flag); break;
  }
  return launch_status();
}

extern "C" int kvc_gather_slots(const void* cache, int64_t block_stride_bytes, int block_size, int64_t num_blocks,
                                int64_t row_bytes, const int64_t* slots, int64_t n, void* out, int32_t* error_flag,
                                void* stream) {
  return slots_launch<true>(cache, nullptr, block_stride_bytes, block_size, num_blocks, row_bytes, slots, n,
                            nullptr, out, error_flag, stream);
}

extern "C" int kvc_scatter_slots(void* cache, int64_t block_stride_bytes, int block_size, int64_t num_blocks,
                                 int64_t row_bytes, const int64_t* slots, int64_t n, const void* in,
                                 int32_t* error_flag, void* stream) {
  return slots_launch<false>(nullptr, cache, block_stride_bytes, block_size, num_blocks, row_bytes, slots, n, in,
                             nullptr, error_flag, stream);
}

extern "C" int kvc_shift_positions(const int64_t* positions, const void* request_indices, int index_bytes,
                                   const int64_t* offsets, int64_t num_offsets, int64_t n, int64_t* out,
                                   int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(positions && request_indices && offsets && out, KVC_ENULL);
  KVC_CHECK_ARG((index_bytes == 4 || index_bytes == 8) && n >= 0 && num_offsets >= 0, KVC_EINVAL);
  if (n == 0) return KVC_OK;
  const unsigned grid = (unsigned)((n + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
  if (index_bytes == 4)
    shift_positions_kernel<int32_t><<<grid, 256, 0, st>>>(positions, (const int32_t*)request_indices, offsets,
                                                          num_offsets, n, out, error_flag);
  else
    shift_positions_kernel<int64_t><<<grid, 256, 0, st>>>(positions, (const int64_t*)request_indices, offsets,
                                                          num_offsets, n, out, error_flag);
  return launch_status();
}

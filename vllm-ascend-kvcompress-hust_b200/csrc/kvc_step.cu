// One compression step behind a single host call (kvc_triattention_run).
//
// The stages call the same validated entry points a caller would call one by
// one, in the same order on the same stream; only the host round trips
// between them go away (one call and one argument block instead of seven).
#include <climits>

#include "kvc_common.cuh"

namespace {

// Block tables of R requests into CSR order: blockIdx.x = request, blockIdx.y = 0
// source / 1 destination.  A table entry is a scheduler page of `bpp`
// consecutive 128-token kernel blocks: kernel block i of the request is
// table[i / bpp] * bpp + i % bpp (bpp = 1: the entries are kernel blocks).
__global__ void gather_tables_kernel(const int64_t* const* __restrict__ src_tables,
                                     const int64_t* __restrict__ src_off, int64_t* src_out,
                                     const int64_t* const* __restrict__ dst_tables,
                                     const int64_t* __restrict__ dst_off, int64_t* dst_out, int bpp) {
  // first kernel of the step, launched in plain stream order; lets the next
  // stage's CTAs onto the SMs early (they wait for this grid in pdl_wait)
  kvc::pdl_trigger();
  const int r = blockIdx.x;
  const int64_t* const* tables = blockIdx.y ? dst_tables : src_tables;
  const int64_t* off = blockIdx.y ? dst_off : src_off;
  int64_t* out = blockIdx.y ? dst_out : src_out;
  const int64_t b = off[r], n = off[r + 1] - b;
  const int64_t* t = tables[r];
  if (bpp == 1) {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[b + i] = __ldg(t + i);
  } else {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[b + i] = __ldg(t + i / bpp) * bpp + i % bpp;
  }
}

// Scheduler page ids -> kernel block ids (one thread per output block).
__global__ void expand_ids_kernel(const int64_t* __restrict__ ids, int64_t n_out, int bpp, int64_t* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_out) out[i] = __ldg(ids + i / bpp) * bpp + i % bpp;
}

int tables_stage(const kvc_triattention_step& s, cudaStream_t st) {
  KVC_CHECK_ARG(s.src_tables && s.src_blocks && s.src_block_off, KVC_ENULL);
  const bool dst = s.dst_tables != nullptr;
  KVC_CHECK_ARG(!dst || (s.dst_blocks && s.dst_block_off), KVC_ENULL);
  KVC_CHECK_ARG(s.cache_blocks_per_page >= 0, KVC_EINVAL);
  if (s.num_requests <= 0) return KVC_OK;
  gather_tables_kernel<<<dim3((unsigned)s.num_requests, dst ? 2 : 1), 128, 0, st>>>(
      s.src_tables, s.src_block_off, s.src_blocks, s.dst_tables, s.dst_block_off, s.dst_blocks,
      s.cache_blocks_per_page > 1 ? s.cache_blocks_per_page : 1);
  return kvc::launch_status();
}

inline void mark(void* const* events, int slot, cudaStream_t st) {
  if (events && events[slot]) cudaEventRecord((cudaEvent_t)events[slot], st);
}

// push: the peer exchange follows, so normalisation delivers each quad's head
// max to the inbox of the rank that owns it instead of writing local rows.
// agg: with one scoring layer, normalisation also writes the aggregate (the
// layer reduction is the identity), so the aggregate stage launches nothing.
int score_stage(const kvc_triattention_step& s, void* const* ev, void* stream, bool push, float* agg) {
  cudaStream_t st = (cudaStream_t)stream;
  const int F = s.rotary_dim / 2;
  const int P = s.head_dim - s.rotary_dim;
  const int heads = s.kv_heads * s.group;
  int rc;
  mark(ev, 0, st);
  const bool tensor = s.scorer == KVC_SCORER_TENSOR || s.scorer == KVC_SCORER_TCGEN05;
  if (tensor) {
    const bool tc05 = s.scorer == KVC_SCORER_TCGEN05;
    rc = (tc05 ? kvc_prepare_score_fragments_tc05 : kvc_prepare_score_fragments)(
        s.omega, s.offsets, s.n_off, s.round_start, s.num_requests, s.score_layers, s.kv_heads, s.group, F, P,
        s.q_real, s.q_imag, s.scale, s.extra, s.q_pass, s.kv_dtype, (uint32_t*)s.score_coef, stream);
    if (rc != KVC_OK) return rc;
    mark(ev, 1, st);
    rc = (tc05 ? kvc_score_paged_keys_tc05 : kvc_score_paged_keys_tc)(
        s.key_maps, s.score_layers, s.kv_dtype, s.num_blocks, s.kv_heads, s.group, s.head_dim, s.rotary_dim,
        s.src_blocks, s.src_block_off, s.tokens, s.page_off, s.num_requests, s.total_pages,
        (const uint32_t*)s.score_coef, s.raw, s.partial, s.error_flag, stream);
  } else if (s.scorer == KVC_SCORER_FMA) {
    rc = kvc_prepare_score_coefficients(s.omega, s.offsets, s.n_off, s.round_start, s.num_requests, s.score_layers,
                                        s.kv_heads, s.group, F, s.q_real, s.q_imag, s.scale, s.extra,
                                        s.score_aggregation, (float*)s.score_coef, stream);
    if (rc != KVC_OK) return rc;
    mark(ev, 1, st);
    rc = kvc_score_paged_keys(s.score_k, s.score_layers, s.kv_dtype, s.block_stride, s.num_blocks, s.kv_heads,
                              s.group, s.head_dim, s.rotary_dim, s.src_blocks, s.src_block_off, s.tokens, s.page_off,
                              s.num_requests, s.total_pages, (const float*)s.score_coef, s.n_off,
                              s.score_aggregation, s.q_pass_t, s.raw, s.partial, s.error_flag, stream);
  } else {
    return KVC_EINVAL;
  }
  if (rc != KVC_OK) return rc;
  mark(ev, 2, st);
  rc = kvc_head_stats(s.partial, s.score_layers, s.num_requests, s.total_pages,
                      tensor ? kvc_tc_partials_per_page() : 1, heads, s.tokens, s.page_off,
                      s.mean, s.var, s.den, stream);
  if (rc != KVC_OK) return rc;
  mark(ev, 3, st);
  if (push) {
    KVC_CHECK_ARG(s.peer_inbox && s.peer_flags, KVC_ENULL);
    return kvc_tp_push_rows(s.raw, s.score_layers, heads, s.total_pages, s.mean, s.den, s.tokens, s.page_off,
                            s.num_requests, s.peer_inbox, s.peer_flags, s.world, s.rank, s.epoch, stream);
  }
  return kvc_normalize_aggregate(s.raw, s.score_layers, heads, s.total_pages, s.mean, s.den, s.tokens, s.page_off,
                                 s.num_requests, s.layer_aggregation, s.rows, agg, stream);
}

}  // namespace

extern "C" int64_t kvc_triattention_step_size(void) { return (int64_t)sizeof(kvc_triattention_step); }

extern "C" int kvc_expand_block_ids(const int64_t* ids, int64_t n_ids, int blocks_per_page, int64_t* out,
                                    void* stream) {
  KVC_CHECK_ARG(ids && out, KVC_ENULL);
  KVC_CHECK_ARG(n_ids >= 0 && blocks_per_page >= 1 && n_ids <= INT64_MAX / blocks_per_page, KVC_EINVAL);
  const int64_t n_out = n_ids * blocks_per_page;
  if (n_out == 0) return KVC_OK;
  expand_ids_kernel<<<(unsigned)((n_out + 255) / 256), 256, 0, (cudaStream_t)stream>>>(ids, n_out, blocks_per_page,
                                                                                         out);
  return kvc::launch_status();
}

extern "C" int kvc_triattention_run(const kvc_triattention_step* step, int stages, void* const* ev, void* stream) {
  KVC_CHECK_ARG(step, KVC_ENULL);
  KVC_CHECK_ARG(stages > 0 && (stages & ~(KVC_STAGE_ALL | KVC_STAGE_EXCHANGE)) == 0, KVC_EINVAL);
  KVC_CHECK_ARG(!((stages & KVC_STAGE_EXCHANGE) && (stages & KVC_STAGE_AGGREGATE)), KVC_EINVAL);
  const kvc_triattention_step& s = *step;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = KVC_OK;
  if (stages & KVC_STAGE_TABLES) {
    rc = tables_stage(s, st);
    if (rc != KVC_OK) return rc;
  }
  const bool fuse_agg = (stages & KVC_STAGE_SCORE) && (stages & KVC_STAGE_AGGREGATE) && s.score_layers == 1;
  if (stages & KVC_STAGE_SCORE) {
    rc = score_stage(s, ev, stream, (stages & KVC_STAGE_EXCHANGE) != 0, fuse_agg ? s.agg : nullptr);
    if (rc != KVC_OK) return rc;
  }
  if (stages & KVC_STAGE_AGGREGATE) {
    mark(ev, 4, st);
    if (!fuse_agg) {
      rc = kvc_aggregate_rows(s.rows, s.score_layers, s.total_pages, s.tokens, s.page_off, s.num_requests,
                              s.layer_aggregation, s.agg, stream);
      if (rc != KVC_OK) return rc;
    }
  }
  if (stages & KVC_STAGE_EXCHANGE) {
    mark(ev, 4, st);
    KVC_CHECK_ARG(s.peer_inbox && s.peer_agg && s.peer_flags, KVC_ENULL);
    rc = kvc_tp_exchange_max(s.peer_inbox, s.peer_agg, s.peer_flags, s.world, s.rank, s.score_layers,
                             s.total_pages, s.tokens, s.page_off, s.num_requests, s.layer_aggregation, s.epoch,
                             s.error_flag, stream);
    if (rc != KVC_OK) return rc;
  }
  if (stages & KVC_STAGE_SELECT) {
    mark(ev, 5, st);
    rc = kvc_select_keep(s.agg, s.tokens, s.page_off, s.num_requests, s.budget, s.prefix, s.recent, s.segments,
                         s.policy, s.keep, s.error_flag, stream);
    if (rc != KVC_OK) return rc;
  }
  if (stages & KVC_STAGE_COMPACT) {
    mark(ev, 6, st);
    // staged rows name scheduler pages: with multi-block pages they are staged
    // after the copy, one entry per page
    const bool pages = s.cache_blocks_per_page > 1;
    rc = kvc_compact(s.k_layers, s.v_layers, s.compact_layers, s.block_stride_bytes, s.num_blocks, s.row_bytes,
                     s.src_blocks, s.src_block_off, s.dst_blocks, s.dst_block_off, s.keep, s.tokens, s.num_requests,
                     s.budget, pages ? nullptr : s.staged_rows, s.staged_row_stride,
                     pages ? nullptr : s.staged_offsets, s.semantic, s.error_flag, stream);
    if (rc != KVC_OK) return rc;
    if (pages && (s.staged_rows || s.staged_offsets)) {
      rc = kvc_stage_commit(s.dst_blocks, s.dst_block_off, s.num_requests, s.cache_blocks_per_page, s.staged_rows,
                            s.staged_row_stride, s.staged_offsets, s.semantic, s.budget, stream);
      if (rc != KVC_OK) return rc;
    }
  }
  mark(ev, 7, st);
  if (s.error_host && s.error_flag && (stages & (KVC_STAGE_SELECT | KVC_STAGE_COMPACT))) {
    if (cudaMemcpyAsync(s.error_host, s.error_flag, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        (s.error_event && cudaEventRecord((cudaEvent_t)s.error_event, st) != cudaSuccess)) {
      cudaGetLastError();
      return KVC_ECUDA;
    }
  }
  return KVC_OK;
}

/*
 * kvc.h -- C ABI of the B200 (sm_100a) TriAttention compression hot path.
 *
 * Library: libkvc_b200.so.  Every entry point
 *   - takes plain device pointers, sizes and a cudaStream_t passed as void*;
 *   - validates its scalar arguments and pointer alignment on the host and
 *     returns a negative KVC_E* status WITHOUT launching when they are bad;
 *   - is asynchronous on the given stream, performs no allocation, no
 *     host<->device copy and no synchronisation;
 *   - reports data-dependent faults found on the device (block id or token
 *     index out of range, budget larger than a request) by OR-ing a KVC_DEV_*
 *     bit into the optional device word `error_flag` and skipping the access.
 *
 * Ragged batches use a page-padded "token space": request r owns the 128-token
 * pages [page_off[r], page_off[r+1]) and the tokens
 * [page_off[r]*128, page_off[r]*128 + tokens[r]) of every per-token buffer.
 * Block tables are CSR: request r's kernel block ids are
 * blocks[block_off[r] .. block_off[r+1]).
 *
 * Paths in the citations below are relative to the reference project
 * vllm-ascend-kvcompress-hust 0.10.0 (src/vllm_ascend_kvcompress/...).
 */
#ifndef KVC_B200_H
#define KVC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVC_ABI_VERSION 1

/* host-side status codes */
#define KVC_OK 0
#define KVC_EINVAL (-22)      /* bad size, count or enum value */
#define KVC_ENULL (-14)       /* required pointer is NULL */
#define KVC_EALIGN (-71)      /* pointer or stride misaligned for the kernel */
#define KVC_EUNSUPPORTED (-95) /* geometry not compiled (e.g. query group > 8) */
#define KVC_ECUDA (-5)        /* the launch itself failed */
#define KVC_ECAPACITY (-28)   /* request larger than a fixed, library-owned scratch */

/* device error bits (OR-ed into *error_flag) */
#define KVC_DEV_BLOCK_RANGE 1   /* a block id outside [0, num_blocks) */
#define KVC_DEV_TOKEN_RANGE 2   /* a keep index outside [0, tokens) */
#define KVC_DEV_BUDGET 4        /* budget/windows impossible for a request */
#define KVC_DEV_TIMEOUT 8       /* a bounded pipeline wait expired (the kernel gave up) */
#define KVC_DEV_INDEX_RANGE 16  /* a request index outside the offsets table */

/* cache element types */
#define KVC_BF16 0
#define KVC_FP16 1

/* aggregation / policy enums */
#define KVC_AGG_MEAN 0
#define KVC_AGG_MAX 1
#define KVC_POLICY_GLOBAL 0
#define KVC_POLICY_V3 1

int kvc_abi_version(void);
const char* kvc_status_string(int status);

/* Floats per (request, scoring layer, kv head) block of `coef`:
 * F * round_up(3*G, 4) for mean aggregation; for max aggregation
 * F * round_up(3*G, 4) + n_off * F * 2 (the per-offset cos/sin table). */
int64_t kvc_coef_floats(int num_freq, int group, int n_off, int aggregation);

/*
 * Phase coefficients of every (request, scoring layer):
 *   c_f = mean_o cos(fp32(offset_o + round_start[r]) * omega[l][f]),
 *   s_f = mean_o sin(...), then per (kv head h, q head g, frequency f)
 *   a = scale*(qr*c - qi*s), b = scale*(qi*c + qr*s), e = extra*scale.
 * Replaces prepare_mean_phase_coefficients (methods/triattention/kernels.py:85-122)
 * and the phase formation of score_post_rope_keys (methods/triattention/scoring.py:77-83),
 * computed directly per request (no angle-addition shortcut).
 * omega [L][F]; q_real, q_imag, scale, extra [L][kvh][G][F] (fp32);
 * offsets [n_off]; round_start [R] (int64, device). coef_out: R*L*kvh*kvc_coef_floats.
 */
int kvc_prepare_score_coefficients(const float* omega, const float* offsets, int n_off,
                                   const int64_t* round_start, int num_requests,
                                   int num_layers, int kv_heads, int group, int num_freq,
                                   const float* q_real, const float* q_imag,
                                   const float* scale, const float* extra,
                                   int aggregation, float* coef_out, void* stream);

/*
 * Raw trigonometric scores of every cached key of every request in every
 * scoring layer, plus per-page partial moments for the per-head statistics.
 * Replaces score_paged_keys_mean_precomputed (methods/triattention/kernels.py:247-317)
 * and the CPU chunk loop of TriAttentionMethod._select_keep_indices
 * (methods/triattention/method.py:405-422), batched over requests and layers.
 *   k_layers     host array [num_layers] of K cache base pointers, each
 *                [num_blocks][128][kv_heads][head_dim] with contiguous inner
 *                dims and `block_stride` elements between blocks.
 *   coef         output of kvc_prepare_score_coefficients (same aggregation).
 *   q_pass_t     [L][kvh][head_dim-rotary_dim][G] fp32 (transposed q_pass_mean),
 *                NULL for full RoPE.
 *   raw_out      [L][total_pages][kvh*G][128] fp32 (page-major: one page's
 *                scores of every query head are one contiguous block).
 *   partial_out  [L][total_pages][kvh*G][2] fp32: (page sum, page sum of
 *                squared deviations from the page mean).
 */
int kvc_score_paged_keys(const void* const* k_layers, int num_layers, int dtype,
                         int64_t block_stride, int64_t num_blocks, int kv_heads, int group,
                         int head_dim, int rotary_dim, const int64_t* src_blocks,
                         const int64_t* src_block_off, const int32_t* tokens,
                         const int32_t* page_off, int num_requests, int total_pages,
                         const float* coef, int n_off, int aggregation, const float* q_pass_t,
                         float* raw_out, float* partial_out, int32_t* error_flag, void* stream);

/*
 * Tensor-core scorer (same contract as kvc_score_paged_keys, mean aggregation):
 * each (page, KV head) K tile is staged by TMA (cp.async.bulk.tensor, 128-byte
 * swizzle) and contracted with mma.sync against hi/lo-split bf16 (or fp16)
 * coefficient fragments.  Replaces score_paged_keys_mean_precomputed
 * (methods/triattention/kernels.py:247-317) for the supported geometries
 * (kvc_tc_supported: query group <= 8 and (rotary/2, head_dim - rotary) in
 * {(64,0), (32,0), (32,192), (32,64), (64,128), (128,0)}).
 *   key_maps     host array of num_layers 128-byte TMA descriptors from
 *                kvc_encode_key_maps (built once per cache binding).
 *   frag         kvc_prepare_score_fragments output: per (request, layer, KV
 *                head) kvc_fragment_words(num_freq, pass_dim) words of 16-bit
 *                coefficients; with an fp16 cache they are scaled by a power of
 *                two (largest magnitude in [2^13, 2^14)) so low-|q| heads keep
 *                their hi/lo split out of fp16's subnormals, and the scorer
 *                undoes the scale exactly.
 *   partial_out  [L][total_pages*parts][kvh*G][2]: (sum, sum of squared
 *                deviations from the partial's mean) per 128/parts-token slice
 *                of each page, parts = kvc_tc_partials_per_page() (the
 *                consumer warps of a CTA, 4).
 */
int kvc_tc_supported(int group, int head_dim, int rotary_dim);
int kvc_tc_partials_per_page(void);
int kvc_encode_key_maps(const void* const* k_layers, int num_layers, int dtype, int64_t block_stride,
                        int64_t num_blocks, int kv_heads, int head_dim, void* maps_out);
int64_t kvc_fragment_words(int num_freq, int pass_dim);
int kvc_prepare_score_fragments(const float* omega, const float* offsets, int n_off,
                                const int64_t* round_start, int num_requests, int num_layers,
                                int kv_heads, int group, int num_freq, int pass_dim,
                                const float* q_real, const float* q_imag, const float* scale,
                                const float* extra, const float* q_pass, int dtype, uint32_t* frag_out,
                                void* stream);
int kvc_score_paged_keys_tc(const void* key_maps, int num_layers, int dtype, int64_t num_blocks,
                            int kv_heads, int group, int head_dim, int rotary_dim,
                            const int64_t* src_blocks, const int64_t* src_block_off,
                            const int32_t* tokens, const int32_t* page_off, int num_requests,
                            int total_pages, const uint32_t* frag, float* raw_out, float* partial_out,
                            int32_t* error_flag, void* stream);

/*
 * The same scorer on the 5th-generation tensor cores (tcgen05): per
 * (page, KV head) tile, M = 128 tokens x N = 16 x K = 16 tcgen05.mma steps
 * with the fp32 accumulator in tensor memory; the rotary band's A operand
 * (kr | ki | m_hi | m_lo) is formed by the CUDA cores into TMEM, the pass band
 * is read from the TMA-staged tile through shared-memory descriptors.  Same
 * arguments, outputs and partials as kvc_score_paged_keys_tc, but its W layout
 * differs: frag must come from kvc_prepare_score_fragments_tc05 (same size,
 * kvc_fragment_words).  Geometries: kvc_tc05_supported (query group <= 8,
 * (rotary/2, head_dim - rotary) in {(64,0), (32,0), (32,192), (32,64),
 * (64,128)}).  One CTA per SM holds all 512 TMEM columns.
 */
int kvc_tc05_supported(int group, int head_dim, int rotary_dim);
int kvc_prepare_score_fragments_tc05(const float* omega, const float* offsets, int n_off,
                                     const int64_t* round_start, int num_requests, int num_layers,
                                     int kv_heads, int group, int num_freq, int pass_dim,
                                     const float* q_real, const float* q_imag, const float* scale,
                                     const float* extra, const float* q_pass, int dtype, uint32_t* frag_out,
                                     void* stream);
int kvc_score_paged_keys_tc05(const void* key_maps, int num_layers, int dtype, int64_t num_blocks,
                              int kv_heads, int group, int head_dim, int rotary_dim,
                              const int64_t* src_blocks, const int64_t* src_block_off,
                              const int32_t* tokens, const int32_t* page_off, int num_requests,
                              int total_pages, const uint32_t* frag, float* raw_out, float* partial_out,
                              int32_t* error_flag, void* stream);

/*
 * Per (scoring layer, request, query head) population mean/variance of the
 * raw scores, combined from the partial moments in fp64; denom = sqrt(max(var, 1e-6)).
 * parts_per_page: 1 (kvc_score_paged_keys) or kvc_tc_partials_per_page()
 * (kvc_score_paged_keys_tc); any divisor of 128.
 * Replaces torch.var_mean(raw, dim=-1, correction=0) (methods/triattention/method.py:379-381,423)
 * and the denominator of normalize_head_scores (methods/triattention/scoring.py:123-128).
 * mean_out, var_out, denom_out: [L][R][kvh*G].
 */
int kvc_head_stats(const float* partial, int num_layers, int num_requests, int total_pages,
                   int parts_per_page, int heads, const int32_t* tokens, const int32_t* page_off,
                   float* mean_out, float* var_out, float* denom_out, void* stream);

/*
 * Normalise (z = (raw - mean) / denom) and take the max over the local query
 * heads, one row per scoring layer: rows_out [L][total_pages*128] (required;
 * also the tensor-parallel all-reduce input).  When agg_out is non-NULL the
 * layers are then reduced (sequential sum then / L, or max) and finalised
 * (NaN -> -inf, +inf -> 1e30) into agg_out [total_pages*128], 16-byte
 * aligned (kvc_aggregate_rows on the same stream; with one layer the
 * normalisation kernel writes agg_out itself).
 * Replaces aggregate_normalized_scores (methods/triattention/kernels.py:407-437),
 * TriAttentionMethod._aggregate_torch (methods/triattention/method.py:477-503)
 * and the finalisation at methods/triattention/method.py:463-467.
 */
int kvc_normalize_aggregate(const float* raw, int num_layers, int heads, int total_pages,
                            const float* mean, const float* denom, const int32_t* tokens,
                            const int32_t* page_off, int num_requests, int layer_aggregation,
                            float* rows_out, float* agg_out, void* stream);

/*
 * Layer reduction of the (all-reduced) per-layer rows and finalisation.
 * Replaces methods/triattention/method.py:458-467 (torch.sum/amax over the
 * TP-synchronised parallel_scores, mean, nan_to_num).
 */
int kvc_aggregate_rows(const float* rows, int num_layers, int total_pages,
                       const int32_t* tokens, const int32_t* page_off, int num_requests,
                       int layer_aggregation, float* agg_out, void* stream);

/*
 * Ragged segmented selection: for every request keep exactly `budget`
 * positions, sorted ascending: the protected prefix and recent windows plus,
 * per V3 segment (or the whole middle for the global policy), the top-quota
 * scores; equal scores are taken lowest position first.
 * Replaces select_keep_indices (methods/triattention/selection.py:108-196,
 * including the batched V3 plan of :24-105).  keep_out [R][budget] int64.
 */
int kvc_select_keep(const float* agg, const int32_t* tokens, const int32_t* page_off,
                    int num_requests, int budget, int prefix, int recent, int segments,
                    int policy, int64_t* keep_out, int32_t* error_flag, void* stream);

/*
 * Compaction of every layer: for each request r and j < budget, copy the K and
 * V rows of token keep[r][j] (through the source block table) into dense
 * position j of the destination block table.  Source and destination blocks
 * must be disjoint (the provider guarantees private destinations).
 * Optionally stages the commit: staged_rows[r][:] = destination block ids,
 * staged_offsets[r] = semantic[r] - budget (the request's position offset).
 * Replaces the per-layer materialize_token_slots loop
 * (methods/triattention/method.py:272-288, methods/triattention/cache.py:9-15,100-111).
 *   k_layers, v_layers  host arrays [num_layers] of cache base pointers.
 *   row_bytes           kv_heads*head_dim*element size (one token, all local heads).
 */
int kvc_compact(const void* const* k_layers, const void* const* v_layers, int num_layers,
                int64_t block_stride_bytes, int64_t num_blocks, int64_t row_bytes,
                const int64_t* src_blocks, const int64_t* src_block_off,
                const int64_t* dst_blocks, const int64_t* dst_block_off, const int64_t* keep,
                const int32_t* tokens, int num_requests, int budget,
                int64_t* staged_rows, int staged_row_stride, int64_t* staged_offsets,
                const int64_t* semantic, int32_t* error_flag, void* stream);

/*
 * Slot gather / scatter through a workspace: out[i] = cache[slot[i]] and
 * cache[slot[i]] = in[i] (slot = block*block_size + within).  Gathering all
 * rows before scattering makes overlapping source/destination slots safe.
 * Replaces _gather_slots/_write_slots/materialize_token_slots
 * (methods/triattention/cache.py:18-45,100-111).
 */
int kvc_gather_slots(const void* cache, int64_t block_stride_bytes, int block_size,
                     int64_t num_blocks, int64_t row_bytes, const int64_t* slots, int64_t n,
                     void* out, int32_t* error_flag, void* stream);
int kvc_scatter_slots(void* cache, int64_t block_stride_bytes, int block_size,
                      int64_t num_blocks, int64_t row_bytes, const int64_t* slots, int64_t n,
                      const void* in, int32_t* error_flag, void* stream);

/*
 * Calibration reduction of pre-RoPE queries q [n_tokens][row_stride] (heads *
 * head_dim used per row): per (head, frequency) sums of re = q[f],
 * im = q[F + f], |.| = sqrt(re^2 + im^2), and per (head, pass dim) sums of
 * q[rotary_dim + p], accumulated (+=) into fp64 outputs.
 * Replaces _LayerAccumulator.add (calibration.py:95-131).
 * workspace: any size of at least 3 * heads * (rotary_dim/2 + head_dim -
 * rotary_dim) doubles (one partial row); kvc_calibration_workspace_doubles()
 * gives the size at which the launch runs at full parallelism on the current
 * device (at most one wave of partial rows, never more than
 * ceil(n_tokens / 512)).  A smaller workspace plans fewer, longer partial rows.
 * The fp32 partials make the last bits of the sums depend on the row count,
 * i.e. on the device and the workspace size; they stay within 1e-6 relative.
 */
int64_t kvc_calibration_workspace_doubles(int64_t n_tokens, int heads, int head_dim,
                                          int rotary_dim);
int kvc_calibration_accumulate(const void* q, int dtype, int64_t n_tokens, int64_t row_stride,
                               int heads, int head_dim, int rotary_dim, double* re_sum,
                               double* im_sum, double* abs_sum, double* pass_sum,
                               double* workspace, int64_t workspace_doubles, void* stream);

/*
 * The same reduction over post-RoPE ("half" style) query rows, undoing the
 * rotation in fp32 registers before summing: row t sits at position
 * first_position + t, theta = fp32(position) * omega[f], and the rotated pair
 * (o1, o2) = (q[f], q[F+f]) of every head counts as
 * (o1 cos + o2 sin, o2 cos - o1 sin).  No rounding back to 16 bits happens
 * between the un-rotation and the sums.  omega [rotary_dim / 2] fp32 (device).
 * No reference counterpart (online calibration from the attention inputs; the
 * reference's stats builder hooks the pre-RoPE projections, calibration.py:197-360).
 */
int kvc_calibration_accumulate_post_rope(const void* q, int dtype, int64_t n_tokens, int64_t row_stride,
                                         int heads, int head_dim, int rotary_dim, int64_t first_position,
                                         const float* omega, double* re_sum, double* im_sum,
                                         double* abs_sum, double* pass_sum, double* workspace,
                                         int64_t workspace_doubles, void* stream);

/*
 * Allocation-free calibration reduction.  No counterpart in the reference: it
 * is an addition of this library for callers that cannot provide device
 * memory -- a process whose GPU memory is already reserved (vLLM sizes the KV
 * cache to the whole memory budget, so a later cudaMalloc may fail) or a
 * foreign-language host that binds only this C ABI without a device allocator.
 * Same inputs, outputs and results (within 1e-6 relative) as
 * kvc_calibration_accumulate; the partial rows live in a library-owned static
 * device array of KVC_CALIB_STATIC_SCRATCH_DOUBLES doubles (8 MiB), which every
 * GPU that loads the library keeps until process exit.  The launch plans only
 * as many partial rows as the array holds, so any token count is served; a
 * head geometry whose one partial row (3 * heads * (rotary_dim/2 + head_dim -
 * rotary_dim) doubles) exceeds the array returns KVC_ECAPACITY without
 * launching.  The first call on each device (and the first after that device's
 * context is reset) looks up the array's device address with
 * cudaGetSymbolAddress; make that first call before any stream capture.  All
 * calls on a device share the array: calls that overlap on the GPU race.  No
 * cudaMalloc/cudaFree or other allocating routine is called.
 */
#define KVC_CALIB_STATIC_SCRATCH_DOUBLES (1 << 20)
int kvc_calibration_accumulate_noalloc(const void* q, int dtype, int64_t n_tokens, int64_t row_stride,
                                       int heads, int head_dim, int rotary_dim, double* re_sum,
                                       double* im_sum, double* abs_sum, double* pass_sum, void* stream);

/*
 * Undo "half"-style RoPE of query rows in place, for statistics gathered from
 * post-RoPE queries (online calibration; no reference counterpart).  Row t sits
 * at position first_position + t; with theta = fp32(position) * omega[f] the
 * rotated pair (o1, o2) = (q[f], q[F+f]) of every head becomes
 * (o1 cos + o2 sin, o2 cos - o1 sin), rounded back to the row's dtype.
 * q [n_tokens][row_stride] BF16/FP16 with heads x head_dim leading elements;
 * omega [rotary_dim / 2] fp32.
 */
int kvc_unrotate_queries(void* q, int dtype, int64_t n_tokens, int64_t row_stride, int heads,
                         int head_dim, int rotary_dim, int64_t first_position, const float* omega,
                         void* stream);

/*
 * Physical decode positions: out[i] = positions[i] - offsets[request_indices[i]].
 * Replaces shift_positions (methods/triattention/kernels.py:35-47).
 * index_bytes: 4 (int32 request indices) or 8 (int64).  An index outside
 * [0, num_offsets) raises KVC_DEV_INDEX_RANGE and passes the position through.
 */
int kvc_shift_positions(const int64_t* positions, const void* request_indices, int index_bytes,
                        const int64_t* offsets, int64_t num_offsets, int64_t n, int64_t* out,
                        int32_t* error_flag, void* stream);

/*
 * Decode-step offsets of compressed requests in one launch:
 *   physical_positions[i] = positions[i] - offsets[request_indices[i]]   (i < num_tokens)
 *   semantic_seq_lens[r] = seq_lens[r]; seq_lens[r] -= offsets[r]        (r < num_reqs)
 * Either part may be empty (num_tokens = 0, or num_reqs = 0 with seq_lens NULL),
 * so a host can shift the slot-mapping positions and, later in the step, the
 * attention lengths.  semantic_seq_lens may be NULL (no copy kept).  Requests
 * never compressed carry offset 0.  Replaces the device work of
 * AscendKVCompressionProvider.physical_positions_for_slot_mapping
 * (provider.py:687-705, i.e. shift_positions, methods/triattention/kernels.py:35-47)
 * and of apply_physical_attention_lengths (provider.py:707-728: the semantic
 * copy and seq_lens.sub_(offsets)); the host-side optimistic lengths stay host work.
 * index_bytes: 4 or 8 (request_indices); len_bytes: 4 or 8 (seq_lens and
 * semantic_seq_lens).  A request index, or a row r, outside [0, num_offsets)
 * raises KVC_DEV_INDEX_RANGE and leaves that value unshifted.
 */
int kvc_decode_offsets(const int64_t* positions, const void* request_indices, int index_bytes,
                       int64_t num_tokens, const int64_t* offsets, int64_t num_offsets,
                       int64_t* physical_positions, void* seq_lens, void* semantic_seq_lens, int len_bytes,
                       int num_reqs, int32_t* error_flag, void* stream);

/*
 * Scheduler pages -> kernel blocks: out[i] = ids[i / blocks_per_page] *
 * blocks_per_page + i % blocks_per_page for i < n_ids * blocks_per_page.
 * Replaces _expand_scheduler_block_ids (provider.py:1273-1287), which turns a
 * 1152- or 2048-token logical page into 9 or 16 consecutive 128-token blocks.
 * (The step below expands inside its block-table gather when
 * kvc_triattention_step.cache_blocks_per_page > 1.)
 */
int kvc_expand_block_ids(const int64_t* ids, int64_t n_ids, int blocks_per_page, int64_t* out, void* stream);

/*
 * Commit staging alone: staged_rows[r][i] = the scheduler page id of request
 * r's i-th destination page (its first kernel block / blocks_per_page; -1 past
 * the request's pages, i < staged_row_stride) and staged_offsets[r] =
 * semantic[r] - budget.  With blocks_per_page = 1 this is the staging that
 * kvc_compact performs.  Replaces the inputs of PendingCompression and of the
 * offset rows (provider.py:38-54, 981-1010).
 */
int kvc_stage_commit(const int64_t* dst_blocks, const int64_t* dst_block_off, int num_requests,
                     int blocks_per_page, int64_t* staged_rows, int staged_row_stride,
                     int64_t* staged_offsets, const int64_t* semantic, int budget, void* stream);

/*
 * Tensor-parallel score sync over NVLink peer memory, replacing the MAX
 * all-reduce of the per-layer rows and the layer reduction after it (the
 * dist.all_reduce(parallel_scores, MAX) of TriAttentionMethod._select_keep_indices
 * and the sum/amax, division and nan_to_num that follow,
 * methods/triattention/method.py:447-467).
 *
 * The step's tokens are split into `world` equal ranges of 4-token quads
 * (kvc_tp_exchange_inbox_floats gives the sizes); rank o owns range o.  Every
 * rank of the TP group calls, once per step and on its stream, with the same
 * world, layers, pages, requests and epoch:
 *   kvc_tp_push_rows     after kvc_head_stats, in place of
 *                        kvc_normalize_aggregate: normalises its local heads'
 *                        raw scores and stores each quad's head max per layer
 *                        into the owning rank's inbox (plain peer stores);
 *   kvc_tp_exchange_max  before the selection: reduces the owned quads from
 *                        its own inbox (max over ranks, NaN-propagating), reduces
 *                        the layers (sequential sum then / L, or max),
 *                        finalises (NaN -> -inf, +inf -> 1e30; page padding 0)
 *                        and stores the scores into every rank's agg buffer.
 * On return (stream order) every rank's agg holds the finalised scores of the
 * whole step, bit-identical to kvc_normalize_aggregate + kvc_aggregate_rows of
 * the TP = 1 rows.  peer_inbox[p] is rank p's inbox
 * (kvc_tp_exchange_inbox_floats(world, L, total_pages) fp32, layout
 * [world source ranks][L][quads per rank][4]), peer_agg[p] its agg buffer
 * ([total_pages*128] fp32) and peer_flags[p] its flag words
 * (kvc_tp_exchange_flag_words(world) int32, zero-initialised once); the three
 * are device arrays of `world` device addresses valid on this GPU (this rank's
 * own buffers at index `rank`, the others mapped with kvc_ipc_open); every
 * inbox/agg buffer 16-byte aligned.
 * epoch: a positive step counter, one larger on every step (flags are never
 * cleared).  Waits for other ranks are bounded (2 s); on expiry the kernel
 * raises KVC_DEV_TIMEOUT in error_flag and completes.  When the exchange has
 * completed on this rank's stream every rank has finished reading its inbox,
 * so the next step's pushes may arrive.  num_layers <= 512.
 * Flag words: delivered[world], pushed[world], two CTA counters, the started
 * epoch, a spare word, then from word kvc_tp_exchange_stamp_word(world)
 * (8-byte aligned when the flags are) four uint64 %globaltimer stamps of this
 * rank's last exchange: first CTA start, first CTA to see every rank's rows
 * delivered, last CTA done, every rank's scores pushed.  Stamp 1 - stamp 0 is
 * the wait for the slowest rank; stamp 3 - stamp 1 the exchange itself.
 */
#define KVC_TP_MAX_WORLD 64
int kvc_tp_exchange_flag_words(int world);
int kvc_tp_exchange_stamp_word(int world);
int64_t kvc_tp_exchange_inbox_floats(int world, int num_layers, int total_pages);
int kvc_tp_push_rows(const float* raw, int num_layers, int heads, int total_pages, const float* mean,
                     const float* denom, const int32_t* tokens, const int32_t* page_off, int num_requests,
                     float* const* peer_inbox, int32_t* const* peer_flags, int world, int rank, int32_t epoch,
                     void* stream);
int kvc_tp_exchange_max(float* const* peer_inbox, float* const* peer_agg, int32_t* const* peer_flags,
                        int world, int rank, int num_layers, int total_pages, const int32_t* tokens,
                        const int32_t* page_off, int num_requests, int layer_aggregation, int32_t epoch,
                        int32_t* error_flag, void* stream);

/*
 * CUDA IPC for the exchange buffers (no reference counterpart; the reference
 * syncs through HCCL).  kvc_ipc_export gives the handle of the allocation that
 * holds `ptr` (KVC_IPC_HANDLE_BYTES) and ptr's offset inside it; another
 * process opens the handle with kvc_ipc_open (base of the allocation on its
 * device) and adds the offset.  Memory from cudaMalloc-backed allocators only
 * (not virtual-memory-managed pools).  kvc_can_access_peer reports whether
 * `device` can load/store `peer`'s memory directly.
 */
#define KVC_IPC_HANDLE_BYTES 64
int kvc_ipc_export(int device, const void* ptr, void* handle_out, int64_t* offset_out);
int kvc_ipc_open(int device, const void* handle, void** base_out);
int kvc_ipc_close(int device, void* base);
int kvc_can_access_peer(int device, int peer);

/*
 * Host helpers (no reference counterpart): record a cudaEvent_t on `stream`,
 * and copy `bytes` between two addresses the CUDA runtime knows (pinned host
 * or device memory, direction inferred) asynchronously on `stream`.  They let a
 * binding stage a step's metadata and arm its error read-back without a
 * framework round trip per call.
 */
int kvc_record_event(void* event, void* stream);
int kvc_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/*
 * One compression step in a single call.
 *
 * No reference counterpart: the reference issues each device op from Python
 * (TriAttentionMethod._select_keep_indices and compress,
 * methods/triattention/method.py:256-475).  The descriptor holds what the
 * entry points above take; the fields under "bound once" are filled when the
 * method binds the KV cache, the rest before each step.  kvc_triattention_run
 * validates and launches the selected stages in order on `stream`, exactly as
 * the individual entry points would, so a step costs one host call instead of
 * seven.  Stages:
 *   KVC_STAGE_TABLES    gather the per-request block tables (src_tables /
 *                       dst_tables: device arrays of device pointers) into
 *                       the CSR arrays src_blocks / dst_blocks, expanding
 *                       scheduler pages into kernel blocks on the way
 *                       (cache_blocks_per_page)
 *   KVC_STAGE_SCORE     prepare fragments/coefficients, score, head stats and
 *                       normalise into rows (kvc_prepare_score_fragments +
 *                       kvc_score_paged_keys_tc, or the FMA pair; kvc_head_stats;
 *                       kvc_normalize_aggregate)
 *   KVC_STAGE_AGGREGATE layer reduction into agg (kvc_aggregate_rows)
 *   KVC_STAGE_SELECT    kvc_select_keep into keep
 *   KVC_STAGE_COMPACT   kvc_compact (+ commit staging when staged_rows/offsets)
 *   KVC_STAGE_EXCHANGE  the tensor-parallel peer score sync with peer_inbox /
 *                       peer_agg / peer_flags, world, rank and epoch: the
 *                       SCORE stage's normalisation becomes kvc_tp_push_rows
 *                       and kvc_tp_exchange_max follows it (agg must be this
 *                       rank's agg buffer of the exchange); not together with
 *                       AGGREGATE
 * A tensor-parallel caller with the peer exchange runs TABLES | SCORE |
 * EXCHANGE | SELECT | COMPACT in one call; with an NCCL all-reduce instead it
 * runs TABLES | SCORE, all-reduces rows with MAX, then AGGREGATE | SELECT | COMPACT.
 * When error_host is set, a call that runs SELECT or COMPACT ends by copying
 * *error_flag to error_host (pinned host memory) and, when error_event is set,
 * recording that cudaEvent_t after the copy, so the host can test the step's
 * device errors later without a synchronisation.  stage_events (optional: KVC_STEP_EVENTS
 * cudaEvent_t handles, NULL entries skipped) are recorded on `stream` before
 * the prepare, score, head-stats, normalise, aggregate, select and compact
 * launches of the stages that run, and after the last launch, for per-stage
 * timing.  Returns the first non-zero status; later stages are not launched.
 */
#define KVC_SCORER_TENSOR 0     /* kvc_score_paged_keys_tc (needs key_maps) */
#define KVC_SCORER_FMA 1        /* kvc_score_paged_keys (needs score_k) */
#define KVC_SCORER_TCGEN05 2    /* kvc_score_paged_keys_tc05 (needs key_maps) */
#define KVC_STAGE_SCORE 1
#define KVC_STAGE_AGGREGATE 2
#define KVC_STAGE_SELECT 4
#define KVC_STAGE_COMPACT 8
#define KVC_STAGE_TABLES 16
#define KVC_STAGE_ALL 31          /* the whole step with tensor parallelism off */
#define KVC_STAGE_EXCHANGE 32     /* the peer score sync (kvc_tp_exchange_max); replaces AGGREGATE */
#define KVC_STEP_EVENTS 8

typedef struct kvc_triattention_step {
  /* bound once */
  int32_t scorer;              /* KVC_SCORER_* */
  int32_t kv_dtype;            /* KVC_BF16 / KVC_FP16 */
  int32_t score_layers;        /* L_s */
  int32_t kv_heads;            /* local KV heads */
  int32_t group;               /* query heads per KV head */
  int32_t head_dim;
  int32_t rotary_dim;
  int32_t n_off;               /* geometric offsets */
  int32_t score_aggregation;   /* KVC_AGG_* over offsets (FMA scorer) */
  int32_t layer_aggregation;   /* KVC_AGG_* over layers */
  int32_t budget;
  int32_t prefix;
  int32_t recent;
  int32_t segments;
  int32_t policy;              /* KVC_POLICY_* */
  int32_t compact_layers;      /* N, every materialised layer */
  int64_t num_blocks;
  int64_t block_stride;        /* elements between blocks (FMA scorer) */
  int64_t block_stride_bytes;
  int64_t row_bytes;           /* kv_heads * head_dim * element size */
  const void* key_maps;        /* [L_s] TMA descriptors (tensor scorer) */
  const void* const* score_k;  /* [L_s] K caches of the scoring layers (FMA scorer) */
  const void* const* k_layers; /* [N] */
  const void* const* v_layers; /* [N] */
  const float* omega;          /* [L_s][F] */
  const float* offsets;        /* [n_off] */
  const float* q_real;         /* [L_s][kvh][G][F] */
  const float* q_imag;
  const float* scale;
  const float* extra;
  const float* q_pass;         /* [L_s][kvh][G][P] or NULL (tensor scorer) */
  const float* q_pass_t;       /* [L_s][kvh][P][G] or NULL (FMA scorer) */
  /* per step */
  int32_t num_requests;
  int32_t total_pages;
  const int32_t* tokens;
  const int32_t* page_off;
  int64_t* src_blocks;         /* CSR by src_block_off; written by KVC_STAGE_TABLES */
  const int64_t* src_block_off;
  int64_t* dst_blocks;         /* CSR by dst_block_off; written by KVC_STAGE_TABLES */
  const int64_t* dst_block_off;
  const int64_t* round_start;
  const int64_t* semantic;
  const int64_t* const* src_tables; /* [R] per-request source tables (KVC_STAGE_TABLES) */
  const int64_t* const* dst_tables; /* [R] destination tables, or NULL */
  /* caller-owned workspaces, sized as for the individual entry points */
  void* score_coef;            /* fragments (tensor) or coefficients (FMA) */
  float* raw;
  float* partial;
  float* mean;
  float* var;
  float* den;
  float* rows;
  float* agg;
  int64_t* keep;
  int64_t* staged_rows;        /* optional commit staging */
  int32_t staged_row_stride;
  int64_t* staged_offsets;
  int32_t* error_flag;
  /* kernel blocks per entry of src_tables / dst_tables (scheduler pages of
   * 128 * cache_blocks_per_page tokens); 0 or 1: the entries are kernel
   * blocks.  Under KVC_STAGE_COMPACT with staging, staged rows then hold
   * scheduler page ids. */
  int32_t cache_blocks_per_page;
  /* optional device-error read-back (see above) */
  int32_t* error_host;
  void* error_event;
  /* KVC_STAGE_EXCHANGE: device arrays of `world` addresses (this rank's at `rank`) */
  float* const* peer_inbox;
  float* const* peer_agg;
  int32_t* const* peer_flags;
  int32_t world;
  int32_t rank;
  int32_t epoch;               /* one larger on every step */
} kvc_triattention_step;

int64_t kvc_triattention_step_size(void);   /* sizeof(kvc_triattention_step), for bindings */
int kvc_triattention_run(const kvc_triattention_step* step, int stages, void* const* stage_events,
                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVC_B200_H */

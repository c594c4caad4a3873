// Decode-step offsets of compressed requests (sm_100a).
//
// After a compression commits, request r's cache holds `budget` physical
// tokens for `semantic` logical ones, so every later step writes its new K/V
// at physical slot = semantic position - offset[r] and attends over
// seq_len - offset[r] tokens, while RoPE keeps the semantic positions.  One
// launch does both parts of a step: threads [0, num_tokens) shift the slot
// positions of the step's tokens, threads past them save each request's
// semantic length and subtract its offset in place.  Rows of requests that
// were never compressed carry offset 0 and pass through unchanged.
#include "kvc_common.cuh"

namespace {

template <typename I, typename S>
__global__ void decode_offsets_kernel(const int64_t* __restrict__ positions, const I* __restrict__ request_indices,
                                      int64_t num_tokens, const int64_t* __restrict__ offsets, int64_t num_offsets,
                                      int64_t* physical_positions, S* seq_lens, S* semantic_seq_lens, int num_reqs,
                                      int32_t* error_flag) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < num_tokens) {
    const int64_t r = (int64_t)request_indices[i];
    if (r < 0 || r >= num_offsets) {
      kvc::raise_flag(error_flag, KVC_DEV_INDEX_RANGE);
      physical_positions[i] = positions[i];
      return;
    }
    physical_positions[i] = positions[i] - __ldg(offsets + r);
    return;
  }
  const int64_t r = i - num_tokens;
  if (r >= num_reqs) return;
  const S len = seq_lens[r];
  if (semantic_seq_lens) semantic_seq_lens[r] = len;
  if (r >= num_offsets) {
    kvc::raise_flag(error_flag, KVC_DEV_INDEX_RANGE);
    return;
  }
  seq_lens[r] = (S)(len - (S)__ldg(offsets + r));
}

template <typename I>
int launch(const int64_t* positions, const void* request_indices, int64_t num_tokens, const int64_t* offsets,
           int64_t num_offsets, int64_t* physical_positions, void* seq_lens, void* semantic_seq_lens, int len_bytes,
           int num_reqs, int32_t* error_flag, cudaStream_t st) {
  const int64_t n = num_tokens + num_reqs;
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (len_bytes == 4)
    decode_offsets_kernel<I, int32_t><<<grid, 256, 0, st>>>(
        positions, (const I*)request_indices, num_tokens, offsets, num_offsets, physical_positions,
        (int32_t*)seq_lens, (int32_t*)semantic_seq_lens, num_reqs, error_flag);
  else
    decode_offsets_kernel<I, int64_t><<<grid, 256, 0, st>>>(
        positions, (const I*)request_indices, num_tokens, offsets, num_offsets, physical_positions,
        (int64_t*)seq_lens, (int64_t*)semantic_seq_lens, num_reqs, error_flag);
  return kvc::launch_status();
}

}  // namespace

extern "C" int kvc_decode_offsets(const int64_t* positions, const void* request_indices, int index_bytes,
                                  int64_t num_tokens, const int64_t* offsets, int64_t num_offsets,
                                  int64_t* physical_positions, void* seq_lens, void* semantic_seq_lens, int len_bytes,
                                  int num_reqs, int32_t* error_flag, void* stream) {
  KVC_CHECK_ARG(offsets, KVC_ENULL);
  KVC_CHECK_ARG(num_tokens >= 0 && num_reqs >= 0 && num_offsets >= 0, KVC_EINVAL);
  KVC_CHECK_ARG(index_bytes == 4 || index_bytes == 8, KVC_EINVAL);
  KVC_CHECK_ARG(len_bytes == 4 || len_bytes == 8, KVC_EINVAL);
  KVC_CHECK_ARG(num_tokens == 0 || (positions && request_indices && physical_positions), KVC_ENULL);
  KVC_CHECK_ARG(num_reqs == 0 || seq_lens, KVC_ENULL);
  if (num_tokens + num_reqs == 0) return KVC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  return index_bytes == 4
             ? launch<int32_t>(positions, request_indices, num_tokens, offsets, num_offsets, physical_positions,
                               seq_lens, semantic_seq_lens, len_bytes, num_reqs, error_flag, st)
             : launch<int64_t>(positions, request_indices, num_tokens, offsets, num_offsets, physical_positions,
                               seq_lens, semantic_seq_lens, len_bytes, num_reqs, error_flag, st);
}

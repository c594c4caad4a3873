"""Torch-facing wrappers of the sm_100a TriAttention kernels (C ABI in include/kvc.h).

Each wrapper checks that its tensors live on a CUDA device with the expected
dtype and layout, passes raw pointers and the current CUDA stream to
``libkvc_b200.so`` and raises RuntimeError on a non-zero status.  There is no
CPU or torch fallback: a non-CUDA tensor is an error.

Correspondence with the reference's device-op layer
(src/vllm_ascend_kvcompress/methods/triattention/kernels.py and the torch ops
of selection.py / cache.py / method.py):

=============================  =====================================================
this module                    reference
=============================  =====================================================
prepare_score_coefficients     prepare_mean_phase_coefficients (kernels.py:85-122),
prepare_score_fragments        phase formation of score_post_rope_keys (scoring.py:77-83)
score_paged_keys(_tc)          score_paged_keys_mean_precomputed (kernels.py:247-317)
head_stats                     torch.var_mean(..., correction=0) (method.py:379,423)
normalize_aggregate            aggregate_normalized_scores (kernels.py:407-437),
                               _aggregate_torch (method.py:477-503), method.py:463-467
aggregate_rows                 method.py:458-467 after the TP all-reduce
select_keep                    select_keep_indices (selection.py:108-196)
compact                        materialize_token_slots per layer (method.py:272-288)
gather_slots / scatter_slots   _gather_slots / _write_slots (cache.py:18-45)
calibration_accumulate         _LayerAccumulator.add (calibration.py:95-131)
shift_positions                shift_positions (kernels.py:35-47)
decode_offsets                 provider.py:687-728 (slot-mapping positions and
                               seq_lens of compressed requests per decode step)
expand_block_ids               _expand_scheduler_block_ids (provider.py:1273-1287)
=============================  =====================================================
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ... import _native as N

BLOCK = 128


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_cur_device = getattr(torch._C, "_cuda_getDevice", None)


def _stream() -> int:
    """The current CUDA stream of the current device, as a raw handle."""
    if _raw_stream is not None and _cur_device is not None:
        return _raw_stream(_cur_device())
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise RuntimeError("the B200 TriAttention kernels require CUDA tensors (no CPU fallback)")


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return N.BF16
    if dtype == torch.float16:
        return N.FP16
    raise RuntimeError(f"unsupported KV/query dtype {dtype}; expected bfloat16 or float16")


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous {dtype} tensor")


_PLAN_FIELDS = ("num_requests", "total_pages", "tokens", "page_off", "src_blocks", "src_off", "dst_blocks",
                "dst_off", "round_start", "semantic", "tokens_host", "max_dst_blocks", "src_tables", "dst_tables",
                "keep_alive", "blocks_per_page")


class BatchPlan:
    """Device metadata of one ragged batch (page-padded token space).

    tokens [R] int32, page_off [R+1] int32, src_blocks/dst_blocks int64 CSR with
    src_off/dst_off [R+1] int64, round_start and semantic [R] int64.  When
    src_tables/dst_tables (device addresses of the per-request block tables,
    int64 [R]) are set, src_blocks/dst_blocks are filled on the device by the
    step's table stage (``gather_tables``) rather than on the host.

    Built either from those tensors (fields in the order above, positional or
    by name), or -- the method's per-step path -- from one staged buffer
    ``meta`` (int64 words ``[page_off | dst_off | round_start | semantic |
    src_tables | dst_tables]`` then int32 words ``[tokens | page_off]``), in
    which case the tensor views are only made when asked for.  The ``*_addr``
    attributes are the device addresses the step descriptor takes.
    """

    def __init__(self, *args, meta: torch.Tensor | None = None, n64: int = 0, with_dst: bool = True, **kw):
        vals = dict(zip(_PLAN_FIELDS, args))
        vals.update(kw)
        self.num_requests = int(vals["num_requests"])
        self.total_pages = int(vals["total_pages"])
        self.src_blocks = vals["src_blocks"]
        self.dst_blocks = vals["dst_blocks"]
        self.tokens_host = tuple(vals["tokens_host"])
        self.max_dst_blocks = int(vals["max_dst_blocks"])
        self.keep_alive = vals.get("keep_alive")
        self.blocks_per_page = int(vals.get("blocks_per_page", 1))
        self.meta = meta
        self.n64 = n64
        R = self.num_requests
        if meta is None:
            self._views = {k: vals.get(k) for k in ("tokens", "page_off", "src_off", "dst_off", "round_start",
                                                    "semantic", "src_tables", "dst_tables")}
            ptr = lambda k: None if self._views[k] is None else self._views[k].data_ptr()
            self.tokens_addr, self.page_off_addr = ptr("tokens"), ptr("page_off")
            self.src_off_addr, self.dst_off_addr = ptr("src_off"), ptr("dst_off")
            self.round_start_addr, self.semantic_addr = ptr("round_start"), ptr("semantic")
            self.src_tables_addr, self.dst_tables_addr = ptr("src_tables"), ptr("dst_tables")
            return
        self._views = None
        base = meta.data_ptr()
        self.src_off_addr = base
        self.dst_off_addr = base + 8 * (R + 1)
        self.round_start_addr = base + 8 * (2 * R + 2)
        self.semantic_addr = base + 8 * (3 * R + 2)
        self.src_tables_addr = base + 8 * (4 * R + 2)
        self.dst_tables_addr = base + 8 * (5 * R + 2) if with_dst else None
        self.tokens_addr = base + 8 * n64
        self.page_off_addr = self.tokens_addr + 4 * R

    def _view(self, name: str, i64_start: int | None, i32_start: int | None, n: int) -> torch.Tensor | None:
        if self._views is not None:
            return self._views[name]
        if i64_start is not None:
            return self.meta[i64_start: i64_start + n]
        return self.meta.view(torch.int32)[2 * self.n64 + i32_start: 2 * self.n64 + i32_start + n]

    @property
    def src_off(self) -> torch.Tensor:
        return self._view("src_off", 0, None, self.num_requests + 1)

    @property
    def dst_off(self) -> torch.Tensor:
        return self._view("dst_off", self.num_requests + 1, None, self.num_requests + 1)

    @property
    def round_start(self) -> torch.Tensor:
        return self._view("round_start", 2 * self.num_requests + 2, None, self.num_requests)

    @property
    def semantic(self) -> torch.Tensor:
        return self._view("semantic", 3 * self.num_requests + 2, None, self.num_requests)

    @property
    def src_tables(self) -> torch.Tensor | None:
        return self._view("src_tables", 4 * self.num_requests + 2, None, self.num_requests)

    @property
    def dst_tables(self) -> torch.Tensor | None:
        if self._views is None and self.dst_tables_addr is None:
            return None
        return self._view("dst_tables", 5 * self.num_requests + 2, None, self.num_requests)

    @property
    def tokens(self) -> torch.Tensor:
        return self._view("tokens", None, 0, self.num_requests)

    @property
    def page_off(self) -> torch.Tensor:
        return self._view("page_off", None, self.num_requests, self.num_requests + 1)

    @property
    def tok_total(self) -> int:
        return self.total_pages * BLOCK


def coef_floats(num_freq: int, group: int, n_off: int, aggregation: int) -> int:
    return int(N.lib().kvc_coef_floats(num_freq, group, n_off, aggregation))


def prepare_score_coefficients(omega, offsets, plan: BatchPlan, q_real, q_imag, scale, extra, aggregation: int,
                               coef_out) -> None:
    require_cuda(omega, offsets, q_real, coef_out)
    L, kvh, G, F = q_real.shape
    for t, n in ((omega, "omega"), (offsets, "offsets"), (q_real, "q_real"), (q_imag, "q_imag"),
                 (scale, "scale"), (extra, "extra"), (coef_out, "coef")):
        _need(t, torch.float32, n)
    N.check(N.lib().kvc_prepare_score_coefficients(
        _p(omega), _p(offsets), offsets.numel(), _p(plan.round_start), plan.num_requests, L, kvh, G, F,
        _p(q_real), _p(q_imag), _p(scale), _p(extra), aggregation, _p(coef_out), _stream()),
        "kvc_prepare_score_coefficients")


def score_paged_keys(k_ptrs, dtype: torch.dtype, block_stride: int, num_blocks: int, kvh: int, group: int,
                     head_dim: int, rotary_dim: int, plan: BatchPlan, coef, n_off: int, aggregation: int,
                     q_pass_t, raw_out, partial_out, error_flag) -> None:
    N.check(N.lib().kvc_score_paged_keys(
        k_ptrs, len(k_ptrs), _dtype_code(dtype), block_stride, num_blocks, kvh, group, head_dim, rotary_dim,
        _p(plan.src_blocks), _p(plan.src_off), _p(plan.tokens), _p(plan.page_off), plan.num_requests,
        plan.total_pages, _p(coef), n_off, aggregation, _p(q_pass_t), _p(raw_out), _p(partial_out),
        _p(error_flag), _stream()), "kvc_score_paged_keys")


def tc_supported(group: int, head_dim: int, rotary_dim: int) -> bool:
    return bool(N.lib().kvc_tc_supported(group, head_dim, rotary_dim))


def tc05_supported(group: int, head_dim: int, rotary_dim: int) -> bool:
    """Geometries of the tcgen05 (TMEM-accumulator) scorer."""
    return bool(N.lib().kvc_tc05_supported(group, head_dim, rotary_dim))


def encode_key_maps(k_ptrs, dtype: torch.dtype, block_stride: int, num_blocks: int, kvh: int, head_dim: int):
    """Host buffer of one 128-byte TMA descriptor per K cache (built once per binding)."""
    import ctypes

    buf = ctypes.create_string_buffer(len(k_ptrs) * N.TENSOR_MAP_BYTES)
    N.check(N.lib().kvc_encode_key_maps(k_ptrs, len(k_ptrs), _dtype_code(dtype), block_stride, num_blocks, kvh,
                                        head_dim, buf), "kvc_encode_key_maps")
    return buf


def fragment_words(num_freq: int, pass_dim: int) -> int:
    return int(N.lib().kvc_fragment_words(num_freq, pass_dim))


def prepare_score_fragments(omega, offsets, plan: BatchPlan, q_real, q_imag, scale, extra, q_pass,
                            dtype: torch.dtype, frag_out, tcgen05: bool = False) -> None:
    """W of the tensor-core scorer (tcgen05=True: the layout kvc_score_paged_keys_tc05 reads)."""
    L, kvh, G, F = q_real.shape
    P = 0 if q_pass is None else q_pass.shape[-1]
    name = "kvc_prepare_score_fragments_tc05" if tcgen05 else "kvc_prepare_score_fragments"
    N.check(getattr(N.lib(), name)(
        _p(omega), _p(offsets), offsets.numel(), _p(plan.round_start), plan.num_requests, L, kvh, G, F, P,
        _p(q_real), _p(q_imag), _p(scale), _p(extra), _p(q_pass), _dtype_code(dtype), _p(frag_out), _stream()),
        name)


def score_paged_keys_tc(key_maps, num_layers: int, dtype: torch.dtype, num_blocks: int, kvh: int, group: int,
                        head_dim: int, rotary_dim: int, plan: BatchPlan, frag, raw_out, partial_out,
                        error_flag, tcgen05: bool = False) -> None:
    name = "kvc_score_paged_keys_tc05" if tcgen05 else "kvc_score_paged_keys_tc"
    N.check(getattr(N.lib(), name)(
        key_maps, num_layers, _dtype_code(dtype), num_blocks, kvh, group, head_dim, rotary_dim,
        _p(plan.src_blocks), _p(plan.src_off), _p(plan.tokens), _p(plan.page_off), plan.num_requests,
        plan.total_pages, _p(frag), _p(raw_out), _p(partial_out), _p(error_flag), _stream()), name)


def head_stats(partial, num_layers: int, heads: int, plan: BatchPlan, mean_out, var_out, den_out,
               parts_per_page: int = 1) -> None:
    N.check(N.lib().kvc_head_stats(
        _p(partial), num_layers, plan.num_requests, plan.total_pages, parts_per_page, heads, _p(plan.tokens),
        _p(plan.page_off), _p(mean_out), _p(var_out), _p(den_out), _stream()), "kvc_head_stats")


def normalize_aggregate(raw, num_layers: int, heads: int, plan: BatchPlan, mean, den, layer_aggregation: int,
                        rows_out=None, agg_out=None) -> None:
    N.check(N.lib().kvc_normalize_aggregate(
        _p(raw), num_layers, heads, plan.total_pages, _p(mean), _p(den), _p(plan.tokens), _p(plan.page_off),
        plan.num_requests, layer_aggregation, _p(rows_out), _p(agg_out), _stream()), "kvc_normalize_aggregate")


def aggregate_rows(rows, num_layers: int, plan: BatchPlan, layer_aggregation: int, agg_out) -> None:
    N.check(N.lib().kvc_aggregate_rows(
        _p(rows), num_layers, plan.total_pages, _p(plan.tokens), _p(plan.page_off), plan.num_requests,
        layer_aggregation, _p(agg_out), _stream()), "kvc_aggregate_rows")


def select_keep(agg, plan: BatchPlan, budget: int, prefix: int, recent: int, segments: int, policy: int,
                keep_out, error_flag) -> None:
    require_cuda(agg, keep_out)
    N.check(N.lib().kvc_select_keep(
        _p(agg), _p(plan.tokens), _p(plan.page_off), plan.num_requests, budget, prefix, recent, segments, policy,
        _p(keep_out), _p(error_flag), _stream()), "kvc_select_keep")


def compact(k_ptrs, v_ptrs, block_stride_bytes: int, num_blocks: int, row_bytes: int, plan: BatchPlan, keep,
            budget: int, error_flag, staged_rows=None, staged_offsets=None) -> None:
    N.check(N.lib().kvc_compact(
        k_ptrs, v_ptrs, len(k_ptrs), block_stride_bytes, num_blocks, row_bytes, _p(plan.src_blocks),
        _p(plan.src_off), _p(plan.dst_blocks), _p(plan.dst_off), _p(keep), _p(plan.tokens), plan.num_requests,
        budget, _p(staged_rows), 0 if staged_rows is None else staged_rows.shape[1], _p(staged_offsets),
        _p(plan.semantic), _p(error_flag), _stream()), "kvc_compact")


def _cache_geometry(cache: torch.Tensor) -> tuple[int, int, int]:
    """(block stride bytes, block size, row bytes) of a [blocks, bs, heads, dim] cache."""
    if cache.ndim != 4:
        raise ValueError("cache must use [blocks, block, heads, dim] layout")
    _, bs, h, d = cache.shape
    es = cache.element_size()
    if cache.stride()[1:] != (h * d, d, 1):
        raise RuntimeError("cache inner dims must be contiguous")
    return cache.stride(0) * es, bs, h * d * es


def gather_slots(cache: torch.Tensor, slots: torch.Tensor, out: torch.Tensor | None = None,
                 error_flag: torch.Tensor | None = None) -> torch.Tensor:
    """``out[i] = cache.view(-1, heads, dim)[slots[i]]`` for any page stride."""
    require_cuda(cache, slots)
    stride_b, bs, row_b = _cache_geometry(cache)
    n = slots.numel()
    if out is None:
        out = torch.empty((n, cache.shape[2], cache.shape[3]), dtype=cache.dtype, device=cache.device)
    _need(slots, torch.int64, "slots")
    if out.dtype != cache.dtype or not out.is_contiguous() or out.numel() * out.element_size() < n * row_b:
        raise RuntimeError("gather output must be a contiguous tensor of the cache dtype and row count")
    N.check(N.lib().kvc_gather_slots(_p(cache), stride_b, bs, cache.shape[0], row_b, _p(slots), n, _p(out),
                                     _p(error_flag), _stream()), "kvc_gather_slots")
    return out


def scatter_slots(cache: torch.Tensor, slots: torch.Tensor, values: torch.Tensor,
                  error_flag: torch.Tensor | None = None) -> None:
    """``cache.view(-1, heads, dim)[slots[i]] = values[i]`` for any page stride."""
    require_cuda(cache, slots, values)
    stride_b, bs, row_b = _cache_geometry(cache)
    _need(slots, torch.int64, "slots")
    if values.dtype != cache.dtype or not values.is_contiguous():
        raise RuntimeError("scatter values must be a contiguous tensor of the cache dtype")
    N.check(N.lib().kvc_scatter_slots(_p(cache), stride_b, bs, cache.shape[0], row_b, _p(slots), slots.numel(),
                                      _p(values), _p(error_flag), _stream()), "kvc_scatter_slots")


def calibration_workspace_doubles(n_tokens: int, heads: int, head_dim: int, rotary_dim: int) -> int:
    return int(N.lib().kvc_calibration_workspace_doubles(n_tokens, heads, head_dim, rotary_dim))


def calibration_accumulate(q: torch.Tensor, heads: int, head_dim: int, rotary_dim: int, re_sum, im_sum,
                           abs_sum, pass_sum, workspace, *, first_position: int | None = None,
                           omega: torch.Tensor | None = None) -> None:
    """Add per-(head, frequency) sums of queries ``q [tokens, >= heads*head_dim]``.

    Pre-RoPE rows by default; with ``first_position`` and ``omega`` the rows are
    post-RoPE at positions ``first_position + t`` and the rotation is undone in
    fp32 inside the reduction (no intermediate 16-bit rounding).
    """
    require_cuda(q, re_sum, workspace, omega)
    if q.ndim != 2 or q.stride(1) != 1:
        raise RuntimeError("calibration queries must be [tokens, width] with a contiguous last dim")
    for t, n in ((re_sum, "re_sum"), (im_sum, "im_sum"), (abs_sum, "abs_sum"), (workspace, "workspace")):
        _need(t, torch.float64, n)
    if (first_position is None) != (omega is None):
        raise ValueError("first_position and omega go together (post-RoPE rows)")
    if omega is None:
        N.check(N.lib().kvc_calibration_accumulate(
            _p(q), _dtype_code(q.dtype), q.shape[0], q.stride(0), heads, head_dim, rotary_dim, _p(re_sum),
            _p(im_sum), _p(abs_sum), _p(pass_sum), _p(workspace), workspace.numel(), _stream()),
            "kvc_calibration_accumulate")
        return
    _need(omega, torch.float32, "omega")
    N.check(N.lib().kvc_calibration_accumulate_post_rope(
        _p(q), _dtype_code(q.dtype), q.shape[0], q.stride(0), heads, head_dim, rotary_dim, int(first_position),
        _p(omega), _p(re_sum), _p(im_sum), _p(abs_sum), _p(pass_sum), _p(workspace), workspace.numel(), _stream()),
        "kvc_calibration_accumulate_post_rope")


def unrotate_queries(q: torch.Tensor, heads: int, head_dim: int, rotary_dim: int, first_position: int,
                     omega: torch.Tensor) -> None:
    """Undo half-style RoPE of ``q`` [n, >= heads*head_dim] (bf16/fp16, CUDA) in place."""
    require_cuda(q, omega)
    if q.ndim != 2 or q.stride(1) != 1:
        raise RuntimeError("unrotate_queries takes [tokens, heads*head_dim] rows with unit inner stride")
    _need(omega, torch.float32, "omega")
    N.check(N.lib().kvc_unrotate_queries(q.data_ptr(), _dtype_code(q.dtype), q.shape[0], q.stride(0), heads,
                                         head_dim, rotary_dim, int(first_position), omega.data_ptr(), _stream()),
            "kvc_unrotate_queries")


def shift_positions(positions: torch.Tensor, request_indices: torch.Tensor, request_offsets: torch.Tensor,
                    output: torch.Tensor, error_flag: torch.Tensor | None = None) -> torch.Tensor:
    """``output = positions - request_offsets[request_indices]`` (reference kernels.py:35-47)."""
    require_cuda(positions, request_indices, request_offsets, output)
    for t, n in ((positions, "positions"), (request_offsets, "request_offsets"), (output, "output")):
        _need(t, torch.int64, n)
    if request_indices.dtype not in (torch.int32, torch.int64) or not request_indices.is_contiguous():
        raise RuntimeError("request_indices must be a contiguous int32/int64 tensor")
    if output.numel() != positions.numel() or request_indices.numel() != positions.numel():
        raise ValueError("positions, request_indices and output must have the same length")
    N.check(N.lib().kvc_shift_positions(
        _p(positions), _p(request_indices), request_indices.element_size(), _p(request_offsets),
        request_offsets.numel(), positions.numel(), _p(output), _p(error_flag), _stream()),
        "kvc_shift_positions")
    return output


def decode_offsets(request_offsets: torch.Tensor, *, positions: torch.Tensor | None = None,
                   request_indices: torch.Tensor | None = None, physical_positions: torch.Tensor | None = None,
                   seq_lens: torch.Tensor | None = None, semantic_seq_lens: torch.Tensor | None = None,
                   num_reqs: int = 0, error_flag: torch.Tensor | None = None) -> None:
    """One launch of the per-step decode offsets (provider.py:687-728).

    ``physical_positions[i] = positions[i] - request_offsets[request_indices[i]]``
    when ``positions`` is given, and for ``r < num_reqs``
    ``semantic_seq_lens[r] = seq_lens[r]; seq_lens[r] -= request_offsets[r]`` when
    ``seq_lens`` is given (in place; int32 or int64).
    """
    require_cuda(request_offsets, positions, request_indices, physical_positions, seq_lens, semantic_seq_lens)
    _need(request_offsets, torch.int64, "request_offsets")
    n = 0
    if positions is not None:
        if request_indices is None or physical_positions is None:
            raise ValueError("positions need request_indices and physical_positions")
        for t, name in ((positions, "positions"), (physical_positions, "physical_positions")):
            _need(t, torch.int64, name)
        if request_indices.dtype not in (torch.int32, torch.int64) or not request_indices.is_contiguous():
            raise RuntimeError("request_indices must be a contiguous int32/int64 tensor")
        n = positions.numel()
        if request_indices.numel() < n or physical_positions.numel() < n:
            raise ValueError("request_indices and physical_positions must cover every position")
    len_bytes = 8
    if seq_lens is not None:
        if seq_lens.dtype not in (torch.int32, torch.int64) or not seq_lens.is_contiguous():
            raise RuntimeError("seq_lens must be a contiguous int32/int64 tensor")
        if semantic_seq_lens is not None and (semantic_seq_lens.dtype != seq_lens.dtype
                                              or not semantic_seq_lens.is_contiguous()):
            raise RuntimeError("semantic_seq_lens must match seq_lens' dtype")
        if num_reqs < 0 or num_reqs > seq_lens.numel() or (
                semantic_seq_lens is not None and num_reqs > semantic_seq_lens.numel()):
            raise ValueError("num_reqs exceeds the length buffers")
        len_bytes = seq_lens.element_size()
    else:
        num_reqs = 0
    N.check(N.lib().kvc_decode_offsets(
        _p(positions), _p(request_indices), request_indices.element_size() if request_indices is not None else 8, n,
        _p(request_offsets), request_offsets.numel(), _p(physical_positions), _p(seq_lens), _p(semantic_seq_lens),
        len_bytes, int(num_reqs), _p(error_flag), _stream()), "kvc_decode_offsets")


def expand_block_ids(ids: torch.Tensor, blocks_per_page: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Scheduler page ids -> consecutive 128-token kernel block ids (provider.py:1273-1287)."""
    require_cuda(ids)
    _need(ids, torch.int64, "ids")
    if blocks_per_page == 1 and out is None:
        return ids
    n = ids.numel() * blocks_per_page
    if out is None:
        out = torch.empty(n, dtype=torch.int64, device=ids.device)
    elif out.dtype != torch.int64 or not out.is_contiguous() or out.numel() < n:
        raise RuntimeError("out must be a contiguous int64 tensor of ids.numel() * blocks_per_page")
    N.check(N.lib().kvc_expand_block_ids(_p(ids), ids.numel(), int(blocks_per_page), _p(out), _stream()),
            "kvc_expand_block_ids")
    return out[:n]

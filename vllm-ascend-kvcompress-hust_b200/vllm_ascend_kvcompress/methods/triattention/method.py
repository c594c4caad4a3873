"""TriAttention token-selection method on B200: score -> select -> compact in CUDA.

Public behaviour follows the reference method
(src/vllm_ascend_kvcompress/methods/triattention/method.py:57-519): the same
name, runtime spec, compatibility check, binding rules (target vs MTP layers,
layer-index checks, TP head sharding of the statistics) and result.  The work
differs in shape: a whole step's requests are processed by one launch per
stage over a ragged, page-padded token space, instead of one torch op chain
per request and per layer, and the stages are issued by one call into the
library (``kvc_triattention_run``):

    gather block tables -> prepare coefficients -> score every page of every
    scoring layer -> per-head moments -> normalise + head max into per-layer
    rows -> layer mean/max (under tensor parallelism: the NVLink peer exchange
    kernel, or one NCCL MAX all-reduce then the layer reduction) -> segmented
    select -> one compaction launch for all layers and requests.

``compress(request)`` is ``compress_many((request,))``; ``compress_many`` is an
optional batched extension a provider may probe for.  All launches go to the
current CUDA stream; nothing here synchronises with the host except the
explicit ``check_device_errors``.
"""

from __future__ import annotations

import ctypes
import os
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from typing import Any

import torch

from ... import _native as N
from ...config import ASCEND_BLOCK_SIZE, JsonScalar
from ..base import (
    CompressionRequest,
    CompressionResult,
    KVCompressionMethod,
    LayerCache,
    MethodRuntimeSpec,
    ModelShape,
    QueryBatchSpan,
    QueryObservation,
)
from . import kernels as K
from .config import TriAttentionConfig
from .scoring import build_geometric_offsets
from .stats import CalibrationStats, DeviceLayerCalibrationStats
from .tp_exchange import PeerScoreExchange, choose_tp_sync_mode

METHOD_NAME = "triattention"
_STRICT_ENV = "KVC_B200_STRICT"
_SCORER_ENV = "KVC_B200_SCORER"


def _queries_per_kv_head(shape: ModelShape) -> int:
    if shape.num_attention_heads % shape.num_kv_heads:
        raise RuntimeError("TriAttention requires query heads divisible by KV heads")
    return shape.num_attention_heads // shape.num_kv_heads


def _is_mtp_cache_layer(layer_name: str) -> bool:
    return ".mtp.layers." in f".{layer_name}."


@dataclass(frozen=True)
class TriAttentionLayerCache:
    name: str
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    stats: DeviceLayerCalibrationStats
    frequency_scale: torch.Tensor | None = None
    extra_coefficient: torch.Tensor | None = None
    offset_cos_mean: torch.Tensor | None = None
    offset_sin_mean: torch.Tensor | None = None


class _Workspaces:
    """Method-owned device buffers, grown (never shrunk) to the largest batch seen."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self._bufs: dict[str, torch.Tensor] = {}
        self._ptrs: dict[str, tuple[int, int]] = {}

    def _buf(self, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
        buf = self._bufs.get(name)
        if buf is None or buf.numel() < numel or buf.dtype != dtype:
            cap = max(numel, int(buf.numel() * 1.25) if buf is not None and buf.dtype == dtype else 0, 1)
            buf = torch.empty(cap + 16, dtype=dtype, device=self.device)
            self._bufs[name] = buf
            self._ptrs[name] = (buf.numel(), buf.data_ptr())
        return buf

    def get(self, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
        return self._buf(name, numel, dtype)[:numel]

    def ptr(self, name: str, numel: int, dtype: torch.dtype) -> int:
        """Device address of the buffer (grown to ``numel`` elements of ``dtype`` if needed)."""
        hit = self._ptrs.get(name)
        if hit is not None and hit[0] >= numel and self._bufs[name].dtype == dtype:
            return hit[1]
        return self._buf(name, numel, dtype).data_ptr()


class _MetadataStager:
    """Per-step request metadata: pinned host ring -> one H2D copy -> device views.

    Each step's integers go into the next of ``slots`` pinned host buffers and
    are copied to the device with a single async copy on the current stream.
    A host buffer is rewritten only after the copy that last read it has
    completed (its event), so the host does not wait for the GPU in steady state.
    """

    def __init__(self, device: torch.device, slots: int = 4) -> None:
        self.device = device
        self.slots = slots
        self.cap = 0
        self.i = 0
        self.host: list[torch.Tensor] = []
        self.events: list[torch.cuda.Event] = []
        self.dev: torch.Tensor | None = None

    def _grow(self, n: int) -> None:
        for ev in self.events:  # old host buffers may still feed a copy
            ev.synchronize()
        cap = max(n, 2 * self.cap, 256)
        self.host = [torch.empty(cap, dtype=torch.int64).pin_memory() for _ in range(self.slots)]
        self.host_np = [h.numpy() for h in self.host]
        self.host_ptr = [h.data_ptr() for h in self.host]
        self.events = []
        for _ in range(self.slots):
            ev = torch.cuda.Event()
            ev.record()  # creates the event (complete once the stream reaches it)
            self.events.append(ev)
        self.event_handles = [ev.cuda_event for ev in self.events]
        self.dev = torch.empty(cap, dtype=torch.int64, device=self.device)
        self.dev_ptr = self.dev.data_ptr()
        self.cap = cap

    def stage(self, i64: list[int], i32: list[int]) -> torch.Tensor:
        """Copy int64 words ``i64`` then int32 words ``i32`` to the device buffer (returned)."""
        n64 = len(i64)
        n = n64 + (len(i32) + 1) // 2
        if n > self.cap:
            self._grow(n)
        slot = self.i
        self.i = (self.i + 1) % self.slots
        self.events[slot].synchronize()  # the copy that last read this host buffer is done
        h = self.host_np[slot]
        h[:n64] = i64
        h.view("int32")[2 * n64: 2 * n64 + len(i32)] = i32
        lib, stream = N.lib(), K._stream()
        N.check(lib.kvc_copy_async(self.dev_ptr, self.host_ptr[slot], 8 * n, stream), "kvc_copy_async")
        N.check(lib.kvc_record_event(self.event_handles[slot], stream), "kvc_record_event")
        return self.dev


class TriAttentionMethod(KVCompressionMethod):
    """TriAttention KV compression with sm_100a kernels."""

    def __init__(self, options: Mapping[str, JsonScalar], vllm_config: Any, model_shape: ModelShape) -> None:
        self.config = TriAttentionConfig.from_method_config(options)
        self.vllm_config = vllm_config
        self.model_shape = model_shape
        self.calibration = CalibrationStats.load(self.config.stats_path)
        self.layer_caches: tuple[TriAttentionLayerCache, ...] = ()
        self.materialization_caches: tuple[LayerCache, ...] = ()
        self.cache_block_size = ASCEND_BLOCK_SIZE
        self.offsets: torch.Tensor | None = None
        self.tensor_parallel_size = 1
        self.tensor_parallel_rank = 0
        self.tp_group = None
        self._peer: PeerScoreExchange | None = None
        self.staged_block_rows: torch.Tensor | None = None
        self.staged_offsets: torch.Tensor | None = None
        # optional timing hooks: .mark(name) records a stage boundary now, .add(name, event)
        # takes an event that the library records at that boundary
        self.profiler = None
        # "auto": tensor-core scorer where the geometry allows, else the CUDA-core one
        self.scorer = "auto"
        self._ws: _Workspaces | None = None
        self._err_host: torch.Tensor | None = None
        self._err_event: torch.cuda.Event | None = None

    # ---- method API v1 ------------------------------------------------------

    @property
    def name(self) -> str:
        return METHOD_NAME

    @property
    def runtime_spec(self) -> MethodRuntimeSpec:
        return MethodRuntimeSpec(
            requires_private_destination=True,
            compression_threshold_tokens=self.config.compression_threshold_tokens,
            required_recompute_tokens=self.config.recompute_window,
            max_physical_num_tokens=self.config.kv_budget,
            min_output_tokens_for_compression=self.config.min_output_tokens_for_compression,
        )

    # ---- online calibration through the query-observation hooks (opt-in) ------

    @property
    def query_window_tokens(self) -> int:
        """Trailing prefill query rows captured per request and scoring layer (0: online calibration off)."""
        return self.config.online_calibration_window

    @property
    def query_layer_indices(self) -> tuple[int, ...] | None:
        """The scoring layers (their statistics are the only ones scoring reads)."""
        if not self.config.online_calibration_window:
            return None
        if self.layer_caches:
            return self._scoring_model_layers
        shape_layers = self.model_shape.full_attention_layer_indices
        return tuple(shape_layers[:: self.config.score_layer_stride])

    def capture_query(self, layer: LayerCache, query: torch.Tensor, spans: tuple[QueryBatchSpan, ...]) -> None:
        """Keep the last ``online_calibration_window`` post-RoPE query rows of each span's request.

        ``query`` is the attention input of one forward, [rows, local heads x head_dim]
        (or [rows, heads, head_dim]); rows of later forwards of the same request
        append to the earlier ones, and only the most recent window is kept.
        """
        W = self.config.online_calibration_window
        slot = self._scoring_slot.get(layer.layer_index) if W else None
        if slot is None:
            return
        width = self.local_kv_heads * self.group * self.head_dim
        rows = query.reshape(query.shape[0], -1)
        if rows.shape[1] != width or rows.dtype not in (torch.bfloat16, torch.float16):
            raise RuntimeError(f"captured query rows must be bf16/fp16 [tokens, {width}] on the bound device")
        for span in spans:
            take = min(span.end - span.start, W)
            if take <= 0:
                continue
            buf, fill = self._observation(span.request_id, rows.dtype)
            have = fill[slot]
            if have + take <= W:
                buf[slot, have:have + take].copy_(rows[span.end - take:span.end])
                fill[slot] = have + take
            else:  # keep the newest W rows, oldest first
                keep = W - take
                if keep:
                    buf[slot, :keep].copy_(buf[slot, have - keep:have].clone())
                buf[slot, keep:W].copy_(rows[span.end - take:span.end])
                fill[slot] = W

    def complete_query_observation(self, observation: QueryObservation) -> None:
        """Reduce the buffered rows with their RoPE undone (positions end at ``semantic_num_tokens``).

        Once a layer has accumulated ``online_calibration_min_tokens`` rows, its
        q_mean_real / q_mean_imag / q_abs_mean (and q_pass_mean) are replaced in
        the scoring tensors by the online means, in place, before the next step.
        """
        entry = self._observations.pop(observation.request_id, None)
        if entry is None:
            return
        buf, fill = entry
        heads = self.local_kv_heads * self.group
        for slot, n in enumerate(fill):
            if n <= 0:
                continue
            # the reduction un-rotates in fp32 registers: no rounding back to 16 bits
            acc = self._online_sums[slot]
            acc.add(buf[slot, :n], heads, self.head_dim, self.rotary_dim,
                    first_position=int(observation.semantic_num_tokens) - n, omega=self.scoring_omega[slot])
            if acc.count >= self.config.online_calibration_min_tokens:
                self._publish_online_stats(slot, acc)
        self._free_buffers.append(buf)

    def discard_query_observation(self, request_id: str) -> None:
        entry = self._observations.pop(request_id, None)
        if entry is not None:
            self._free_buffers.append(entry[0])

    def _observation(self, request_id: str, dtype: torch.dtype):
        entry = self._observations.get(request_id)
        if entry is None:
            L, W = self.scoring_layer_count, self.config.online_calibration_window
            shape = (L, W, self.local_kv_heads * self.group * self.head_dim)
            buf = next((b for b in self._free_buffers if b.dtype == dtype), None)
            if buf is not None:
                self._free_buffers.remove(buf)
            else:
                buf = torch.empty(shape, dtype=dtype, device=self.offsets.device)
            entry = self._observations[request_id] = (buf, [0] * L)
        return entry

    def _publish_online_stats(self, slot: int, acc) -> None:
        """Online means of one scoring layer -> its scoring tensors (same addresses)."""
        kvh, G, F = self.local_kv_heads, self.group, self.num_freq
        n = float(acc.count)
        qr = (acc.real_sum / n).float().view(kvh, G, F)
        qi = (acc.imag_sum / n).float().view(kvh, G, F)
        qa = (acc.abs_sum / n).float().view(kvh, G, F)
        self.scoring_q_real[slot].copy_(qr)
        self.scoring_q_imag[slot].copy_(qi)
        self.scoring_extra[slot].copy_(qa - torch.sqrt(qr.square() + qi.square() + 1e-8))
        if self.pass_dim and acc.pass_sum is not None:
            qp = (acc.pass_sum / n).float().view(kvh, G, self.pass_dim)
            if self.scoring_q_pass is not None:
                self.scoring_q_pass[slot].copy_(qp)
            self.scoring_q_pass_t[slot].copy_(qp.transpose(-1, -2))
        self.online_published[slot] = acc.count

    def compatibility_reasons(self, worker: Any) -> tuple[str, ...]:
        del worker
        return self.calibration.validate(self.model_shape)

    def bind_model_runner(self, runner: Any, layer_caches: tuple[LayerCache, ...]) -> None:
        device = torch.device(runner.device)
        if device.type != "cuda":
            raise RuntimeError("the B200 TriAttention method requires CUDA KV caches")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        K.require_cuda(*(c.k_cache for c in layer_caches))
        N.lib()  # fail at bind time if the native library is missing
        self.tensor_parallel_size = int(self.vllm_config.parallel_config.tensor_parallel_size)
        self.tensor_parallel_rank = 0
        self._peer = None
        if self.tensor_parallel_size > 1:
            self.tp_group, self.tensor_parallel_rank = self._resolve_tp_group(runner)
            self._peer = self._bind_peer_exchange(device)
        stats = self.calibration.to_device(
            self.model_shape, device, tensor_parallel_rank=self.tensor_parallel_rank,
            tensor_parallel_size=self.tensor_parallel_size)
        self.offsets = build_geometric_offsets(int(self.vllm_config.model_config.max_model_len), device)
        mtp = tuple(c for c in layer_caches if _is_mtp_cache_layer(c.name))
        targets = tuple(c for c in layer_caches if not _is_mtp_cache_layer(c.name))
        spec = getattr(self.vllm_config, "speculative_config", None)
        if mtp and (len(mtp) != 1 or mtp[0].name != "mtp.layers.0.self_attn.attn"
                    or getattr(spec, "method", None) != "mtp"
                    or getattr(spec, "num_speculative_tokens", None) != 2):
            raise RuntimeError("uncalibrated MTP cache requires Qwen3.5 MTP2")
        if len(targets) != len(self.model_shape.full_attention_layer_indices):
            raise RuntimeError("allocated full-attention layer count does not match calibration")
        bound, seen = [], set()
        self._model_layer_of = {c.name: c.layer_index for c in targets}
        for c in targets:
            if c.layer_index not in stats:
                raise RuntimeError(f"attention layer {c.name!r} resolves to invalid model layer index {c.layer_index}")
            if c.layer_index in seen:
                raise RuntimeError(f"multiple cache layers resolve to model layer index {c.layer_index}")
            seen.add(c.layer_index)
            st = stats[c.layer_index]
            qmag = torch.sqrt(st.q_mean_real.square() + st.q_mean_imag.square() + 1e-8)
            bound.append(TriAttentionLayerCache(
                name=c.name, k_cache=c.k_cache, v_cache=c.v_cache, stats=st,
                frequency_scale=torch.sqrt(st.freq_scale_sq), extra_coefficient=st.q_abs_mean - qmag))
        if seen != set(self.model_shape.full_attention_layer_indices):
            raise RuntimeError("allocated target full-attention layers do not match calibration: "
                               f"allocated={sorted(seen)} expected={sorted(self.model_shape.full_attention_layer_indices)}")
        self.layer_caches = tuple(bound)
        self.materialization_caches = layer_caches
        self._bind_geometry(device)
        self._bind_scoring_tensors()
        self._ws = _Workspaces(device)
        self._stager = _MetadataStager(device)
        self._err = torch.zeros(1, dtype=torch.int32, device=device)
        self._err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._err_event = None
        # the native step copies the error word to _err_host and records this
        # event after every selecting call, so a later call can test it cheaply
        self._err_ev = torch.cuda.Event()
        self._err_ev.record()  # creates the event
        self._results: tuple | None = None
        self._strict = os.environ.get(_STRICT_ENV, "") == "1"
        self._last_shape = (0, 0, 0, 0)
        self._bind_step()
        self._bind_online_calibration()

    def compress(self, request: CompressionRequest) -> CompressionResult:
        return self.compress_many((request,))[0]

    # ---- batched extension ----------------------------------------------------

    def compress_many(self, requests: Sequence[CompressionRequest], *, stage_commit: bool = False,
                      cache_blocks_per_page: int = 1) -> tuple[CompressionResult, ...]:
        """Score, select and compact a whole step's requests with one launch per stage.

        ``cache_blocks_per_page > 1``: the requests' device block tables hold
        scheduler page ids, each page being that many consecutive 128-token
        kernel blocks (the provider's 1152/2048-token logical pages); the
        pages are expanded on the device while the tables are gathered, and
        with ``stage_commit`` the staged rows hold page ids.
        """
        reqs = tuple(requests)
        if not reqs:
            return ()
        self._require_bound()
        self._raise_pending_device_error()
        plan = self._plan([(r.physical_num_tokens, r.semantic_num_tokens, r.source_block_ids_device,
                            r.destination_block_ids_device) for r in reqs], bpp=cache_blocks_per_page)
        self._run_step(plan, compact=True, stage_commit=stage_commit)
        self._err_event = self._err_ev  # recorded by the native step behind its error read-back
        if self._strict:
            self.check_device_errors()
        if self._results is None or len(self._results) < len(reqs):
            lengths = tuple((c.name, self.config.kv_budget) for c in self.materialization_caches)
            one = CompressionResult(physical_num_tokens=self.config.kv_budget, per_layer_physical_num_tokens=lengths)
            self._results = (one,) * max(len(reqs), 2 * len(self._results or ()))  # immutable: shared
        return self._results[: len(reqs)]

    def select_many(self, requests: Sequence[CompressionRequest], *, cache_blocks_per_page: int = 1
                    ) -> torch.Tensor:
        """Keep indices ``[R, kv_budget]`` (int64, sorted per row) without compaction."""
        reqs = tuple(requests)
        self._require_bound()
        plan = self._plan([(r.physical_num_tokens, r.semantic_num_tokens, r.source_block_ids_device,
                            r.destination_block_ids_device) for r in reqs], need_destination=False,
                          bpp=cache_blocks_per_page)
        self._run_step(plan, compact=False)
        return self._keep_view(len(reqs)).view(len(reqs), self.config.kv_budget).clone()

    def _select_keep_indices(self, source_block_ids: torch.Tensor, physical_num_tokens: int,
                             round_start: int) -> torch.Tensor:
        """Sorted keep positions of one request (the reference method's private hook)."""
        self._require_bound()
        plan = self._plan([(physical_num_tokens, round_start, source_block_ids, None)], need_destination=False)
        self._run_step(plan, compact=False)
        return self._keep_view(1).clone()

    def check_device_errors(self) -> None:
        """Synchronise on the last launch and raise if a kernel reported a bad index."""
        if self._ws is None:
            return
        torch.cuda.current_stream().synchronize()
        bits = int(self._err.item())
        self._err_event = None
        self._err_host.zero_()
        if bits:
            self._err.zero_()
            raise RuntimeError(self._describe_error(bits))

    # ---- binding helpers ----------------------------------------------------

    def _resolve_tp_group(self, runner: Any):
        """TP group and rank: vLLM's, unless the runner carries ``kvc_tp_group``/``kvc_tp_rank``.

        The override lets a host that does not initialise vLLM's parallel state
        (a standalone engine, a benchmark) pass its own process group and rank.
        """
        group = getattr(runner, "kvc_tp_group", None)
        rank = getattr(runner, "kvc_tp_rank", None)
        if rank is not None:
            return group, int(rank)
        if group is not None:
            import torch.distributed as dist

            return group, dist.get_rank(group)
        from vllm.distributed import get_tp_group

        tp = get_tp_group()
        return tp.device_group, int(tp.rank_in_group)

    def _bind_online_calibration(self) -> None:
        from ...calibration import LayerAccumulator

        scoring = self.layer_caches[:: self.config.score_layer_stride]
        self._scoring_model_layers = tuple(self._model_layer_of[c.name] for c in scoring)
        self._scoring_slot = {idx: i for i, idx in enumerate(self._scoring_model_layers)}
        self._observations: dict[str, tuple[torch.Tensor, list[int]]] = {}
        self._free_buffers: list[torch.Tensor] = []
        self._online_sums = [LayerAccumulator() for _ in scoring]
        self.online_published = [0] * len(scoring)

    def _bind_peer_exchange(self, device: torch.device):
        """Peer-memory score sync when the TP group is an NCCL group of GPUs that can reach each other."""
        import torch.distributed as dist

        group = self.tp_group
        if group is None or not dist.is_initialized() or dist.get_backend(group) != "nccl":
            return None
        if choose_tp_sync_mode(group, device.index) != "peer":
            return None
        return PeerScoreExchange(group, self.tensor_parallel_rank, self.tensor_parallel_size, device)

    def _bind_geometry(self, device: torch.device) -> None:
        caches = self.materialization_caches
        k0 = self.layer_caches[0].k_cache
        if k0.ndim != 4 or k0.shape[1] != ASCEND_BLOCK_SIZE:
            raise RuntimeError("TriAttention requires 128-token kernel cache blocks")
        self.cache_block_size = int(k0.shape[1])
        nb, _, kvh, d = k0.shape
        expected_kvh = self.model_shape.num_kv_heads // self.tensor_parallel_size
        if kvh != expected_kvh:
            raise RuntimeError("local KV-cache head count does not match tensor-parallel model shape: "
                               f"expected {expected_kvh}, got {kvh}")
        if k0.dtype not in (torch.bfloat16, torch.float16):
            raise RuntimeError(f"unsupported KV cache dtype {k0.dtype}")
        for c in caches:
            for t in (c.k_cache, c.v_cache):
                if t.device != device or t.dtype != k0.dtype:
                    raise RuntimeError(f"layer {c.name!r} cache must be {k0.dtype} on {device}")
                if tuple(t.shape) != tuple(k0.shape) or t.stride() != k0.stride():
                    raise RuntimeError(f"layer {c.name!r} cache geometry differs from the first layer")
                if t.stride()[1:] != (kvh * d, d, 1) or t.stride(0) < ASCEND_BLOCK_SIZE * kvh * d:
                    raise RuntimeError(f"layer {c.name!r} cache must have contiguous inner blocks")
        es = k0.element_size()
        self.kv_dtype = k0.dtype
        self.num_blocks = int(nb)
        self.local_kv_heads = int(kvh)
        self.head_dim = int(d)
        self.block_stride = int(k0.stride(0))
        self.block_stride_bytes = self.block_stride * es
        self.row_bytes = kvh * d * es
        self._k_all = N.pointer_array([c.k_cache.data_ptr() for c in caches])
        self._v_all = N.pointer_array([c.v_cache.data_ptr() for c in caches])

    def _bind_scoring_tensors(self) -> None:
        layers = self.layer_caches[:: self.config.score_layer_stride]
        self.scoring_layer_count = len(layers)
        self._k_score = N.pointer_array([c.k_cache.data_ptr() for c in layers])
        st0 = layers[0].stats
        self.group = _queries_per_kv_head(self.model_shape)
        self.rotary_dim = int(st0.rotary_dim or self.head_dim)
        self.num_freq = self.rotary_dim // 2
        self.pass_dim = self.head_dim - self.rotary_dim
        if self.pass_dim and any(c.stats.q_pass_mean is None for c in layers):
            raise RuntimeError("partial-RoPE scoring requires q_pass_mean")
        if any(c.stats.rope_style != "half" for c in layers):
            raise RuntimeError("the CUDA scorer supports the 'half' RoPE layout only")
        stack = lambda f: torch.stack([f(c) for c in layers]).contiguous()
        self.scoring_omega = stack(lambda c: c.stats.omega)
        self.scoring_q_real = stack(lambda c: c.stats.q_mean_real)
        self.scoring_q_imag = stack(lambda c: c.stats.q_mean_imag)
        self.scoring_scale = stack(lambda c: c.frequency_scale)
        self.scoring_extra = stack(lambda c: c.extra_coefficient)
        # [L][kvh][P][G]: one unrotated dim's G coefficients are contiguous
        self.scoring_q_pass_t = (stack(lambda c: c.stats.q_pass_mean).transpose(-1, -2).contiguous()
                                 if self.pass_dim else None)
        self.score_aggregation_code = N.AGG_MEAN if self.config.score_aggregation == "mean" else N.AGG_MAX
        self.layer_aggregation_code = N.AGG_MEAN if self.config.layer_aggregation == "mean" else N.AGG_MAX
        self.coef_block = K.coef_floats(self.num_freq, self.group, self.offsets.numel(), self.score_aggregation_code)
        choice = os.environ.get(_SCORER_ENV, self.scorer)
        if choice not in ("auto", "tensor", "tcgen05", "fma"):
            raise ValueError(f"{_SCORER_ENV} must be auto, tensor, tcgen05 or fma")
        supported = K.tc05_supported if choice == "tcgen05" else K.tc_supported
        tc_ok = (self.config.score_aggregation == "mean"
                 and supported(self.group, self.head_dim, self.rotary_dim)
                 and (self.block_stride * 2) % 16 == 0)
        if choice in ("tensor", "tcgen05") and not tc_ok:
            raise RuntimeError(f"the {choice} scorer does not support this geometry/aggregation")
        self.use_tensor_scorer = tc_ok and choice != "fma"
        # "auto"/"tensor": the mma.sync kernel (measured faster on this contraction);
        # "tcgen05": the TMEM-accumulator kernel
        self.use_tcgen05 = self.use_tensor_scorer and choice == "tcgen05"
        if self.use_tensor_scorer:
            self._key_maps = K.encode_key_maps(self._k_score, self.kv_dtype, self.block_stride, self.num_blocks,
                                               self.local_kv_heads, self.head_dim)
            self.scoring_q_pass = stack(lambda c: c.stats.q_pass_mean) if self.pass_dim else None
            self.frag_block = K.fragment_words(self.num_freq, self.pass_dim)
            self._tc_parts = int(N.lib().kvc_tc_partials_per_page())

    # ---- per-step pipeline ----------------------------------------------------

    def _require_bound(self) -> None:
        if self.offsets is None or not self.layer_caches or self._ws is None:
            raise RuntimeError("TriAttention method is not bound to KV cache")

    def _plan(self, items, need_destination: bool = True, bpp: int = 1) -> K.BatchPlan:
        """Validate a batch on the host and stage its metadata on the device.

        The per-request block tables are not copied here: their device
        addresses travel with the metadata and the step's first stage gathers
        them into the CSR arrays ``src_blocks`` / ``dst_blocks`` (expanding
        scheduler pages of ``bpp`` kernel blocks).
        """
        budget = self.config.kv_budget
        bs = self.cache_block_size
        dev_index = self.offsets.get_device()
        i64_t = torch.int64
        if isinstance(bpp, bool) or not isinstance(bpp, int) or bpp < 1:
            raise ValueError("cache_blocks_per_page must be a positive integer")
        tokens, sem, src_ptrs, dst_ptrs, keep_alive = [], [], [], [], []
        page_off = [0]
        dst_need = -(-budget // bs)
        dst_min = -(-dst_need // bpp)
        for t, s, src, dst in items:
            t, s = int(t), int(s)
            if budget <= 0 or budget > t:
                raise ValueError("budget must be in [1, token_count]")
            n = -(-t // bs)
            if src.numel() < -(-n // bpp):
                raise RuntimeError("source block table is shorter than the physical token count")
            if src.dtype is not i64_t or src.get_device() != dev_index or not src.is_contiguous():
                src = src.to(device=self.offsets.device, dtype=i64_t).contiguous()
                keep_alive.append(src)
            tokens.append(t)
            page_off.append(page_off[-1] + n)
            sem.append(s)
            src_ptrs.append(src.data_ptr())
            if need_destination:
                if dst is None or dst.numel() < dst_min:
                    raise RuntimeError("destination block table is shorter than kv_budget")
                if dst.dtype is not i64_t or dst.get_device() != dev_index or not dst.is_contiguous():
                    dst = dst.to(device=self.offsets.device, dtype=i64_t).contiguous()
                    keep_alive.append(dst)
                dst_ptrs.append(dst.data_ptr())
        R = len(tokens)
        dst_off = list(range(0, (R + 1) * dst_need, dst_need)) if need_destination else [0] * (R + 1)
        i64 = page_off + dst_off + sem + sem + src_ptrs + dst_ptrs
        meta = self._stager.stage(i64, tokens + page_off)
        ws = self._ws
        src_blocks = ws.get("src_blocks", page_off[-1], i64_t)
        dst_blocks = ws.get("dst_blocks", R * dst_need, i64_t) if need_destination else src_blocks[:0]
        return K.BatchPlan(num_requests=R, total_pages=page_off[-1], meta=meta, n64=len(i64),
                           src_blocks=src_blocks, dst_blocks=dst_blocks, tokens_host=tuple(tokens),
                           max_dst_blocks=dst_need, with_dst=need_destination, keep_alive=keep_alive,
                           blocks_per_page=bpp)

    def _mark(self, name: str) -> None:
        if self.profiler is not None:
            self.profiler.mark(name)

    def _bind_step(self) -> None:
        """Fill the bound-once fields of the native step descriptor."""
        cfg = self.config
        st = N.TriAttentionStep()
        st.scorer = (N.SCORER_TCGEN05 if self.use_tcgen05 else
                     N.SCORER_TENSOR if self.use_tensor_scorer else N.SCORER_FMA)
        st.kv_dtype = K._dtype_code(self.kv_dtype)
        st.score_layers = self.scoring_layer_count
        st.kv_heads = self.local_kv_heads
        st.group = self.group
        st.head_dim = self.head_dim
        st.rotary_dim = self.rotary_dim
        st.n_off = self.offsets.numel()
        st.score_aggregation = self.score_aggregation_code
        st.layer_aggregation = self.layer_aggregation_code
        st.budget = cfg.kv_budget
        st.prefix = cfg.protected_prefix_window
        st.recent = cfg.protected_recent_window
        st.segments = cfg.position_segments
        st.policy = N.POLICY_V3 if cfg.position_policy == "v3" else N.POLICY_GLOBAL
        st.compact_layers = len(self.materialization_caches)
        st.num_blocks = self.num_blocks
        st.block_stride = self.block_stride
        st.block_stride_bytes = self.block_stride_bytes
        st.row_bytes = self.row_bytes
        if self.use_tensor_scorer:
            st.key_maps = ctypes.addressof(self._key_maps)
            st.q_pass = K._p(self.scoring_q_pass)
        st.score_k = ctypes.addressof(self._k_score)
        st.k_layers = ctypes.addressof(self._k_all)
        st.v_layers = ctypes.addressof(self._v_all)
        st.omega = self.scoring_omega.data_ptr()
        st.offsets = self.offsets.data_ptr()
        st.q_real = self.scoring_q_real.data_ptr()
        st.q_imag = self.scoring_q_imag.data_ptr()
        st.scale = self.scoring_scale.data_ptr()
        st.extra = self.scoring_extra.data_ptr()
        st.q_pass_t = K._p(self.scoring_q_pass_t)
        st.error_flag = self._err.data_ptr()
        st.error_host = self._err_host.data_ptr()
        st.error_event = self._err_ev.cuda_event
        self._step = st
        self._step_ref = ctypes.byref(st)

    def _launch(self, stages: int, slots, exchange: bool = False) -> None:
        """kvc_triattention_run on the current stream (with stage events when profiled)."""
        events = None
        prof = self.profiler
        if prof is not None and getattr(prof, "active", True):
            events = (ctypes.c_void_p * N.STEP_EVENTS)()
            for i in slots:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()  # creates the event; the library records it again at its stage boundary
                events[i] = ev.cuda_event
                prof.add("tp_sync" if exchange and i == 4 else N.STEP_EVENT_NAMES[i], ev)
        N.check(N.lib().kvc_triattention_run(self._step_ref, stages, events, K._stream()), "kvc_triattention_run")

    def _set_plan(self, plan: K.BatchPlan) -> N.TriAttentionStep:
        """Point the step descriptor at one batch's device metadata."""
        st = self._step
        st.num_requests = plan.num_requests
        st.total_pages = plan.total_pages
        st.tokens = plan.tokens_addr
        st.page_off = plan.page_off_addr
        st.src_blocks = plan.src_blocks.data_ptr()
        st.src_block_off = plan.src_off_addr
        st.dst_blocks = plan.dst_blocks.data_ptr()
        st.dst_block_off = plan.dst_off_addr
        st.round_start = plan.round_start_addr
        st.semantic = plan.semantic_addr
        st.src_tables = plan.src_tables_addr
        st.dst_tables = plan.dst_tables_addr
        st.cache_blocks_per_page = plan.blocks_per_page
        return st

    def _gather_tables(self, plan: K.BatchPlan) -> None:
        """Fill plan.src_blocks / plan.dst_blocks on the device (the step's table stage alone)."""
        self._set_plan(plan)
        N.check(N.lib().kvc_triattention_run(self._step_ref, N.STAGE_TABLES, None, K._stream()),
                "kvc_triattention_run")

    def _run_step(self, plan: K.BatchPlan, *, compact: bool, stage_commit: bool = False) -> None:
        """Score, select and (optionally) compact one batch (keep indices land in the "keep" workspace)."""
        ws = self._ws
        L = self.scoring_layer_count
        heads = self.local_kv_heads * self.group
        R, tok = plan.num_requests, plan.tok_total
        parts = self._tc_parts if self.use_tensor_scorer else 1
        st = self._set_plan(plan)
        f32, i64 = torch.float32, torch.int64
        if self.use_tensor_scorer:
            st.score_coef = ws.ptr("frag", R * L * self.local_kv_heads * self.frag_block, torch.int32)
        else:
            st.score_coef = ws.ptr("coef", R * L * self.local_kv_heads * self.coef_block, f32)
        st.raw = ws.ptr("raw", L * heads * tok, f32)
        st.partial = ws.ptr("partial", L * plan.total_pages * parts * heads * 2, f32)
        st.mean = ws.ptr("mean", L * R * heads, f32)
        st.var = ws.ptr("var", L * R * heads, f32)
        st.den = ws.ptr("den", L * R * heads, f32)
        st.rows = ws.ptr("rows", L * tok, f32)
        st.agg = ws.ptr("agg", tok, f32)
        st.keep = ws.ptr("keep", R * self.config.kv_budget, i64)
        self._last_shape = (L, R, heads, tok)
        staged_rows = staged_off = None
        row_len = -(-plan.max_dst_blocks // plan.blocks_per_page)  # staged entries are scheduler pages
        if compact and stage_commit:
            staged_rows = ws.get("staged_rows", R * row_len, torch.int64).view(R, row_len)
            staged_off = ws.get("staged_off", R, torch.int64)
        st.staged_rows = K._p(staged_rows)
        st.staged_row_stride = row_len
        st.staged_offsets = K._p(staged_off)
        tail = N.STAGE_AGGREGATE | N.STAGE_SELECT | (N.STAGE_COMPACT if compact else 0)
        tail_slots = (4, 5, 6, 7) if compact else (4, 5, 7)
        head = N.STAGE_TABLES | N.STAGE_SCORE
        ex = self._peer
        if ex is not None:
            # normalisation pushes each rank's rows into the owners' inboxes and
            # the exchange kernel replaces the all-reduce and the layer reduction,
            # inside the same native call as the other stages
            ex.ensure(L, tok)
            st.agg = ex.agg_ptr
            st.peer_inbox, st.peer_agg, st.peer_flags = ex.tables()
            st.world, st.rank = ex.world, ex.rank
            st.epoch = ex.next_epoch()
            stages = head | N.STAGE_EXCHANGE | (tail & ~N.STAGE_AGGREGATE)
            self._launch(stages, (0, 1, 2, 3, *tail_slots), exchange=True)
            if self.profiler is not None and hasattr(self.profiler, "exchange_done"):
                self.profiler.exchange_done(ex)
        elif self.tensor_parallel_size > 1:
            self._launch(head, (0, 1, 2, 3))
            self._mark("tp_sync")
            self._tp_all_reduce_max(ws.get("rows", L * tok, f32))
            self._launch(tail, tail_slots)
        else:
            self._launch(head | tail, (0, 1, 2, 3, *tail_slots))
        if compact:
            self.staged_block_rows, self.staged_offsets = staged_rows, staged_off

    @property
    def last_stats(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        """(raw, mean, var, agg) workspace views of the last step, for inspection and tests."""
        L, R, heads, tok = self._last_shape
        ws = self._ws
        agg = self._peer.agg_view(tok) if self._peer is not None else ws.get("agg", tok, torch.float32)
        return (ws.get("raw", L * heads * tok, torch.float32), ws.get("mean", L * R * heads, torch.float32),
                ws.get("var", L * R * heads, torch.float32), agg)

    def _keep_view(self, R: int) -> torch.Tensor:
        return self._ws.get("keep", R * self.config.kv_budget, torch.int64)

    def _tp_all_reduce_max(self, rows: torch.Tensor) -> None:
        tp_score_sync(rows, self.tp_group)

    @property
    def tp_sync_mode(self) -> str:
        """"peer" (NVLink exchange kernel), "nccl" (MAX all-reduce) or "none" (TP=1)."""
        if self.tensor_parallel_size == 1:
            return "none"
        return "peer" if self._peer is not None else "nccl"

    # ---- device error reporting ---------------------------------------------

    def _raise_pending_device_error(self) -> None:
        ev = self._err_event
        if ev is not None and ev.query():
            bits = int(self._err_host.item())
            self._err_event = None
            if bits:
                self._err.zero_()
                raise RuntimeError(self._describe_error(bits))

    @staticmethod
    def _describe_error(bits: int) -> str:
        what = []
        if bits & N.DEV_BLOCK_RANGE:
            what.append("a block id outside the KV cache")
        if bits & N.DEV_TOKEN_RANGE:
            what.append("a keep index outside its request")
        if bits & N.DEV_BUDGET:
            what.append("a request shorter than kv_budget or its protected windows")
        if bits & N.DEV_TIMEOUT:
            what.append("a pipeline wait that timed out")
        if bits & N.DEV_INDEX_RANGE:
            what.append("a request index outside the offsets table")
        return "TriAttention kernels rejected " + ", ".join(what)


def tp_score_sync(rows: torch.Tensor, group=None) -> None:
    """Tensor-parallel score sync: one in-place MAX all-reduce of the per-layer rows.

    ``rows`` holds every scoring layer's head-max row of every request of the
    step (``[L_s, tokens]``), so a step issues one collective.  MAX commutes
    with KV-head sharding, hence every rank ends with the TP=1 rows and selects
    identical indices (reference method.py:447-461 issues the same MAX per
    request).  ``group`` defaults to vLLM's tensor-parallel device group.
    """
    import torch.distributed as dist

    if group is None:
        from vllm.distributed import get_tp_group

        group = get_tp_group().device_group
    dist.all_reduce(rows, op=dist.ReduceOp.MAX, group=group)


def create_triattention_method(options: Mapping[str, JsonScalar], vllm_config: Any,
                               model_shape: ModelShape) -> KVCompressionMethod:
    return TriAttentionMethod(options, vllm_config, model_shape)


# Backward-compatible import name from the pre-registry layout.
TriAttentionAscendConfig = TriAttentionConfig

"""Worker-side step adapter around the hot path: plans -> one batched call -> commit -> decode offsets.

This is the part of the reference's worker provider
(src/vllm_ascend_kvcompress/provider.py, ``AscendKVCompressionProvider``)
that sits on the compression hot path and runs every step:

* ``compress_scheduled_requests`` (provider.py:471-601): the same eligibility
  rules per scheduled request (a scheduler plan, not already pending, output
  limit, final-prefill or current-physical-window length, threshold, block
  table and private-destination checks), then -- where the reference calls
  ``method.compress`` once per request -- ONE ``compress_many`` call for the
  whole step when the method offers it, with the scheduler pages expanded into
  128-token kernel blocks on the device and the commit rows staged by the
  library; methods without ``compress_many`` get the reference's per-request
  loop.  Results become ``PendingCompression`` entries.
* ``before_update_states`` (provider.py:321-371): commit a pending result on the
  request's next scheduled step (block-table row swap, ``ActiveCompression``).
* ``after_update_states`` / ``sync_request_offset_rows`` (provider.py:460-469,
  981-1010): the per-request offset rows, copied to the device when they change.
* ``physical_positions_for_slot_mapping`` and ``apply_physical_attention_lengths``
  (provider.py:687-728): the per-decode-step offsets, through ``kvc_decode_offsets``.

The runner is duck-typed like the reference's tests do it (``device``,
``requests``, ``input_batch``, ``req_indices``, ``seq_lens``,
``optimistic_seq_lens_cpu``, ``max_num_reqs``, ``max_num_tokens``).  What is
vLLM/Ascend binding rather than step work -- cache discovery, compatibility
checks, graph-mode and hybrid (GDN) metadata, MTP, query-capture plumbing --
is not part of this adapter.
"""

from __future__ import annotations

import inspect
from dataclasses import dataclass
from typing import Any

import torch

from .config import KERNEL_BLOCK_SIZE
from .methods.base import CompressionRequest, CompressionResult, MethodRuntimeSpec
from .methods.triattention import kernels as K
from .transaction import PLAN_ATTRIBUTE


@dataclass(frozen=True)
class PendingCompression:
    """A compacted request waiting for its commit step (provider.py:36-42)."""

    semantic_anchor: int
    physical_anchor: int
    block_ids: tuple[int, ...]
    per_layer_physical_num_tokens: tuple[tuple[str, int], ...] | None = None


@dataclass(frozen=True)
class ActiveCompression:
    """A committed request: its semantic -> physical offset (provider.py:45-54)."""

    semantic_anchor: int
    physical_anchor: int
    per_layer_physical_num_tokens: tuple[tuple[str, int], ...] | None = None

    @property
    def removed_tokens(self) -> int:
        return self.semantic_anchor - self.physical_anchor


def request_max_tokens(request: Any) -> int:
    """The request's output limit, as the reference reads it (provider.py:1255-1266)."""
    value = getattr(request, "max_tokens", None)
    if value is None:
        value = getattr(getattr(request, "sampling_params", None), "max_tokens", None)
    if value is None and getattr(request, "pooling_params", None) is not None:
        value = 1
    if isinstance(value, bool) or not isinstance(value, int) or value < 0:
        raise RuntimeError("current vLLM worker request must expose a non-negative output limit")
    return value


def expand_scheduler_block_ids(block_ids, blocks_per_page: int, device) -> torch.Tensor:
    """Scheduler page ids -> consecutive 128-token kernel block ids (provider.py:1273-1287).

    On CUDA the expansion is one ``kvc_expand_block_ids`` launch; a host-side
    runner (the reference's own unit-test form) gets the same ids from torch.
    """
    ids = torch.as_tensor(block_ids, dtype=torch.long, device=device)
    if blocks_per_page == 1:
        return ids
    if ids.device.type == "cuda":
        return K.expand_block_ids(ids.contiguous(), blocks_per_page)
    return (ids.unsqueeze(1) * blocks_per_page + torch.arange(blocks_per_page, dtype=torch.long)).reshape(-1)


class BatchedCompressionProvider:
    """The per-step worker loop of the compression hot path (see the module docstring)."""

    def __init__(self, method: Any, runner: Any, *, runtime_spec: MethodRuntimeSpec | None = None,
                 attention_group_index: int = 0, scheduler_block_size: int = KERNEL_BLOCK_SIZE,
                 cache_block_size: int = KERNEL_BLOCK_SIZE, layer_names: tuple[str, ...] | None = None,
                 pin_memory: bool | None = None) -> None:
        if scheduler_block_size % cache_block_size:
            raise RuntimeError("scheduler block size must be a multiple of the kernel block size")
        self.method = method
        self.runner = runner
        self.runtime_spec = runtime_spec if runtime_spec is not None else method.runtime_spec
        self.attention_group_index = attention_group_index
        self.scheduler_block_size = scheduler_block_size
        self.cache_block_size = cache_block_size
        self.cache_blocks_per_scheduler_block = scheduler_block_size // cache_block_size
        self.layer_names = layer_names
        self.pending: dict[str, PendingCompression] = {}
        self.active: dict[str, ActiveCompression] = {}
        device = torch.device(getattr(runner, "device", "cpu"))
        self.device = device
        pin = device.type == "cuda" if pin_memory is None else pin_memory
        max_reqs = int(getattr(runner, "max_num_reqs", 0) or 0)
        max_tokens = int(getattr(runner, "max_num_tokens", 0) or 0)
        self._request_offsets_cpu = torch.zeros(max_reqs, dtype=torch.int64, pin_memory=pin)
        self._request_offsets_device = torch.zeros(max_reqs, dtype=torch.int64, device=device)
        self._physical_positions = torch.empty(max_tokens, dtype=torch.int64, device=device)
        self._semantic_seq_lens_device: torch.Tensor | None = None
        self._semantic_seq_lens_cpu: torch.Tensor | None = None
        self._offset_row_snapshot: tuple[int, ...] = ()
        self._has_active_rows = False
        self._physical_lengths_applied = False
        self._tables_host: torch.Tensor | None = None
        self._tables_dev: torch.Tensor | None = None
        self._tables_event = self._offsets_event = None
        self._error = torch.zeros(1, dtype=torch.int32, device=device) if device.type == "cuda" else None
        batched = getattr(method, "compress_many", None)
        self._batched = batched if callable(batched) else None
        self._batched_pages = self._batched is not None and "cache_blocks_per_page" in inspect.signature(
            self._batched).parameters
        self.last_batch_size = 0

    # ---- compression transactions ---------------------------------------------

    def compress_scheduled_requests(self, scheduler_output: Any) -> None:
        """Run the scheduler-authorised transactions of this step (after the attention forward)."""
        if self.runner is None:
            raise RuntimeError("KV compression provider is not cache-bound")
        spec = self.runtime_spec
        plans = getattr(scheduler_output, PLAN_ATTRIBUTE, {})
        required = -(-spec.max_physical_num_tokens // self.scheduler_block_size)
        batch = []
        for request_id, scheduled in scheduler_output.num_scheduled_tokens.items():
            plan = plans.get(request_id)
            if plan is None or request_id in self.pending:
                continue
            request = self.runner.requests.get(request_id)
            if request is None:
                continue
            if request_max_tokens(request) < spec.min_output_tokens_for_compression:
                continue
            semantic = int(request.num_computed_tokens) + int(scheduled)
            active = self.active.get(request_id)
            if active is None:
                physical = semantic
                if semantic != int(request.num_prompt_tokens):
                    continue
            else:
                physical = active.physical_anchor + semantic - active.semantic_anchor
            if semantic != plan.semantic_anchor:
                raise RuntimeError(f"request {request_id!r} semantic length disagrees with the scheduler "
                                   "compression plan")
            if physical < spec.compression_threshold_tokens:
                continue
            if self.attention_group_index >= len(request.block_ids):
                raise RuntimeError("request has no full-attention block table")
            source_ids = tuple(int(v) for v in request.block_ids[self.attention_group_index])
            if len(source_ids) < required:
                raise RuntimeError(f"request {request_id!r} has too few blocks for compression")
            if source_ids != plan.source_block_ids:
                raise RuntimeError(f"request {request_id!r} source block table disagrees with the scheduler "
                                   "compression plan")
            destination_ids = tuple(plan.destination_block_ids)
            if len(destination_ids) != required or set(destination_ids) & set(source_ids):
                raise RuntimeError(f"request {request_id!r} requires private destination blocks")
            per_layer = None
            if active is not None and active.per_layer_physical_num_tokens is not None:
                per_layer = tuple((name, length + semantic - active.semantic_anchor)
                                  for name, length in active.per_layer_physical_num_tokens)
            batch.append((request_id, semantic, physical, source_ids, destination_ids, plan, per_layer))
        self.last_batch_size = len(batch)
        if not batch:
            return
        if self._batched is not None:
            results = self._compress_batched(batch)
        else:
            results = [self._compress_one(item) for item in batch]
        for (request_id, semantic, _, _, destination_ids, _, _), result in zip(batch, results):
            compacted = result.physical_num_tokens
            if isinstance(compacted, bool) or not isinstance(compacted, int):
                raise RuntimeError("method returned a non-integer physical length")
            if compacted != spec.max_physical_num_tokens:
                raise RuntimeError(f"method {self.method.name!r} returned unexpected length {compacted}")
            per_layer = self._validate_per_layer_lengths(result.per_layer_physical_num_tokens, compacted)
            self.pending[request_id] = PendingCompression(semantic, compacted, destination_ids, per_layer)

    def _compress_batched(self, batch) -> tuple[CompressionResult, ...]:
        """One method call for the step: every request's scheduler pages in one H2D copy."""
        bpp = self.cache_blocks_per_scheduler_block
        on_device = self._batched_pages or bpp == 1
        flat = [v for item in batch for v in item[3]] + [v for item in batch for v in item[4]]
        n = len(flat)
        self._host_copy_done("_tables_event")  # the previous step's copy has read the host buffer
        if self._tables_host is None or self._tables_host.numel() < n:
            cap = max(n, 2 * (self._tables_host.numel() if self._tables_host is not None else 0), 256)
            self._tables_host = torch.empty(cap, dtype=torch.int64, pin_memory=self.device.type == "cuda")
            self._tables_dev = torch.empty(cap, dtype=torch.int64, device=self.device)
        self._tables_host[:n] = torch.tensor(flat, dtype=torch.int64)
        dev = self._tables_dev[:n]
        dev.copy_(self._tables_host[:n], non_blocking=True)
        self._host_copy_issued("_tables_event")
        sizes = [len(item[3]) for item in batch] + [len(item[4]) for item in batch]
        views = list(torch.split(dev, sizes))
        if not on_device:  # a batched method that takes kernel blocks only
            views = [expand_scheduler_block_ids(v, bpp, self.device) for v in views]
        R = len(batch)
        reqs = [CompressionRequest(
            request_id=rid, semantic_num_tokens=sem, physical_num_tokens=phys, source_block_ids=(src,),
            destination_block_ids=(dst,), source_block_ids_device=views[j], destination_block_ids_device=views[R + j],
            plan=plan, per_layer_physical_num_tokens=per_layer)
            for j, (rid, sem, phys, src, dst, plan, per_layer) in enumerate(batch)]
        kwargs = {"stage_commit": True}
        if self._batched_pages:
            kwargs["cache_blocks_per_page"] = bpp
        return tuple(self._batched(reqs, **kwargs))

    def _compress_one(self, item) -> CompressionResult:
        """The reference's per-request call, for methods without ``compress_many``."""
        rid, sem, phys, src, dst, plan, per_layer = item
        bpp = self.cache_blocks_per_scheduler_block
        return self.method.compress(CompressionRequest(
            request_id=rid, semantic_num_tokens=sem, physical_num_tokens=phys, source_block_ids=(src,),
            destination_block_ids=(dst,),
            source_block_ids_device=expand_scheduler_block_ids(src, bpp, self.device),
            destination_block_ids_device=expand_scheduler_block_ids(dst, bpp, self.device),
            plan=plan, per_layer_physical_num_tokens=per_layer))

    def _validate_per_layer_lengths(self, lengths, maximum: int):
        """provider.py:603-633: positive lengths <= the group maximum, one per bound layer."""
        if lengths is None:
            return None
        if not isinstance(lengths, tuple):
            raise RuntimeError("per-layer physical lengths must be a tuple")
        values: dict[str, int] = {}
        for entry in lengths:
            if not isinstance(entry, tuple) or len(entry) != 2:
                raise RuntimeError("per-layer physical lengths must be (name, length) pairs")
            name, length = entry
            if name in values:
                raise RuntimeError("per-layer physical lengths repeat a layer")
            if isinstance(length, bool) or not isinstance(length, int) or not 0 < length <= maximum:
                raise RuntimeError("per-layer physical lengths must be positive and <= group maximum")
            values[name] = length
        names = self.layer_names if self.layer_names is not None else tuple(values)
        if set(values) != set(names) or len(values) != len(names):
            raise RuntimeError("per-layer physical lengths omit a full-attention layer")
        return tuple((name, values[name]) for name in names)

    def _host_copy_issued(self, name: str) -> None:
        if self.device.type == "cuda":
            ev = getattr(self, name, None) or torch.cuda.Event()
            ev.record()
            setattr(self, name, ev)

    def _host_copy_done(self, name: str) -> None:
        ev = getattr(self, name, None)
        if ev is not None:
            ev.synchronize()

    # ---- commit and offsets -------------------------------------------------------

    def before_update_states(self, scheduler_output: Any) -> None:
        """Commit the previous step's results on their requests' next scheduled step."""
        reset = set(getattr(scheduler_output, "finished_req_ids", ()))
        reset.update(getattr(scheduler_output, "preempted_req_ids", ()) or ())
        cached = getattr(scheduler_output, "scheduled_cached_reqs", None)
        reset.update(getattr(cached, "resumed_req_ids", ()) or ())
        for request_id in reset:
            self.pending.pop(request_id, None)
            self.active.pop(request_id, None)
        for request_id, pending in tuple(self.pending.items()):
            if request_id not in scheduler_output.num_scheduled_tokens:
                continue
            request = self.runner.requests.get(request_id)
            if request is None:
                self.pending.pop(request_id, None)
                continue
            tables = list(request.block_ids)
            tables[self.attention_group_index] = list(pending.block_ids)
            request.block_ids = tuple(tables)
            batch = self.runner.input_batch
            row = batch.req_id_to_index.get(request_id)
            if row is not None:
                batch.block_table.add_row(request.block_ids, row)
            self.active[request_id] = ActiveCompression(pending.semantic_anchor, pending.physical_anchor,
                                                        pending.per_layer_physical_num_tokens)
            self.pending.pop(request_id, None)

    def after_update_states(self, scheduler_output: Any) -> None:
        del scheduler_output
        live = self.runner.requests.keys()
        for request_id in (self.pending.keys() | self.active.keys()) - live:
            self.pending.pop(request_id, None)
            self.active.pop(request_id, None)
        self._physical_lengths_applied = False
        self.sync_request_offset_rows()

    def sync_request_offset_rows(self) -> None:
        """Per-row semantic - physical offsets of the batch, copied to the device when they change."""
        batch = self.runner.input_batch
        num_reqs = int(batch.num_reqs)
        offsets = tuple(self.active[r].removed_tokens if r in self.active else 0 for r in batch.req_ids[:num_reqs])
        if offsets == self._offset_row_snapshot:
            return
        rows = max(len(self._offset_row_snapshot), num_reqs)
        if rows > self._request_offsets_cpu.numel():
            raise RuntimeError("batch has more requests than the runner's max_num_reqs")
        self._host_copy_done("_offsets_event")  # the previous copy has read the pinned rows
        self._request_offsets_cpu[:rows].zero_()
        if offsets:
            self._request_offsets_cpu[:num_reqs] = torch.tensor(offsets, dtype=torch.int64)
        self._request_offsets_device[:rows].copy_(self._request_offsets_cpu[:rows], non_blocking=True)
        self._host_copy_issued("_offsets_event")
        self._offset_row_snapshot = offsets
        self._has_active_rows = any(offsets)

    def physical_positions_for_slot_mapping(self, positions: torch.Tensor) -> torch.Tensor:
        """Slot-mapping positions of this step's tokens minus their request's offset (RoPE keeps ``positions``)."""
        if not self._has_active_rows:
            return positions
        n = positions.numel()
        if n > self._physical_positions.numel():
            raise RuntimeError("step has more tokens than the runner's max_num_tokens")
        out = self._physical_positions[:n]
        K.decode_offsets(self._request_offsets_device, positions=positions.reshape(-1),
                         request_indices=self.runner.req_indices.gpu[:n], physical_positions=out,
                         error_flag=self._error)
        return out

    def apply_physical_attention_lengths(self) -> None:
        """Attention lengths of compressed requests in physical space (after host sampling decisions)."""
        if self._physical_lengths_applied or not self._has_active_rows:
            return
        num_reqs = int(self.runner.input_batch.num_reqs)
        seq_lens = self.runner.seq_lens
        if self._semantic_seq_lens_device is None or self._semantic_seq_lens_device.numel() < seq_lens.numel() \
                or self._semantic_seq_lens_device.dtype != seq_lens.dtype:
            self._semantic_seq_lens_device = torch.empty_like(seq_lens)
        K.decode_offsets(self._request_offsets_device, seq_lens=seq_lens,
                         semantic_seq_lens=self._semantic_seq_lens_device, num_reqs=num_reqs, error_flag=self._error)
        cpu = self.runner.optimistic_seq_lens_cpu
        if self._semantic_seq_lens_cpu is None or self._semantic_seq_lens_cpu.numel() < cpu.numel() \
                or self._semantic_seq_lens_cpu.dtype != cpu.dtype:
            self._semantic_seq_lens_cpu = torch.empty_like(cpu)
        self._semantic_seq_lens_cpu[:num_reqs].copy_(cpu[:num_reqs])
        cpu[:num_reqs].sub_(self._request_offsets_cpu[:num_reqs].to(cpu.dtype))
        self._physical_lengths_applied = True

    @property
    def semantic_seq_lens(self) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        """(device, host) semantic lengths saved by the last ``apply_physical_attention_lengths``."""
        return self._semantic_seq_lens_device, self._semantic_seq_lens_cpu

    def check_device_errors(self) -> None:
        """Raise if a decode-offset launch met a request index outside the offsets table."""
        if self._error is None:
            return
        torch.cuda.current_stream(self.device).synchronize()
        bits = int(self._error.item())
        if bits:
            self._error.zero_()
            raise RuntimeError("kvc_decode_offsets met a request index outside the offsets table")

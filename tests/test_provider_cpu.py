"""The provider-shaped step adapter on the CPU, with recording methods and a fake runner.

The cases restate the reference's worker-provider tests
(tests/test_provider_integration.py of the reference: final-prefill arming,
private destinations, repeated compression windows, the short-output skip,
the commit step, the page expansion) for ``BatchedCompressionProvider``, plus
the batched path: one ``compress_many`` call per step carrying every eligible
request, with scheduler pages handed over unexpanded when the method takes the
expansion factor.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from vllm_ascend_kvcompress.methods.base import CompressionRequest, CompressionResult, MethodRuntimeSpec
from vllm_ascend_kvcompress.provider import (
    ActiveCompression,
    BatchedCompressionProvider,
    PendingCompression,
    expand_scheduler_block_ids,
)
from vllm_ascend_kvcompress.transaction import PLAN_ATTRIBUTE, CompressionPlan


class _Recording:
    """A v1 method without the batched extension (the per-request loop)."""

    name = "recording"
    runtime_spec = MethodRuntimeSpec(True, 256, 128, 128)

    def __init__(self, per_layer=None) -> None:
        self.requests: list[CompressionRequest] = []
        self.per_layer = per_layer

    def compress(self, request: CompressionRequest) -> CompressionResult:
        self.requests.append(request)
        return CompressionResult(physical_num_tokens=128, per_layer_physical_num_tokens=self.per_layer)


class _Batched(_Recording):
    """A method with ``compress_many`` that takes scheduler pages."""

    def __init__(self) -> None:
        super().__init__()
        self.calls: list[tuple[tuple[CompressionRequest, ...], dict]] = []

    def compress_many(self, requests, *, stage_commit=False, cache_blocks_per_page=1):
        reqs = tuple(requests)
        self.calls.append((reqs, {"stage_commit": stage_commit, "cache_blocks_per_page": cache_blocks_per_page}))
        return tuple(CompressionResult(physical_num_tokens=128) for _ in reqs)


class _BlockTable:
    def __init__(self) -> None:
        self.added = None

    def add_row(self, block_ids, row) -> None:
        self.added = block_ids, row


def _runner(**requests):
    return SimpleNamespace(device=torch.device("cpu"), requests=requests, max_num_reqs=4, max_num_tokens=16,
                           input_batch=SimpleNamespace(req_id_to_index={k: i for i, k in enumerate(requests)},
                                                       req_ids=list(requests), num_reqs=len(requests),
                                                       block_table=_BlockTable()))


def _output(plans: dict, scheduled: dict) -> SimpleNamespace:
    out = SimpleNamespace(num_scheduled_tokens=scheduled, finished_req_ids=set(), preempted_req_ids=set(),
                          scheduled_cached_reqs=SimpleNamespace(resumed_req_ids=set()))
    setattr(out, PLAN_ATTRIBUTE, plans)
    return out


def _request(computed=256, prompt=300, max_tokens=128, blocks=(2, 0, 3)):
    return SimpleNamespace(num_computed_tokens=computed, num_prompt_tokens=prompt, max_tokens=max_tokens,
                           block_ids=(list(blocks),))


def test_final_prefill_compresses_and_arms_worker_commit():
    method = _Recording()
    p = BatchedCompressionProvider(method, _runner(r=_request()))
    p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0, 3), (50,))}, {"r": 44}))
    assert p.pending["r"] == PendingCompression(300, 128, (50,))
    (req,) = method.requests
    assert req.physical_num_tokens == 300 and req.semantic_num_tokens == 300
    assert req.source_block_ids == ((2, 0, 3),) and req.destination_block_ids == ((50,),)
    assert req.source_block_ids_device.tolist() == [2, 0, 3]


def test_batched_method_gets_one_call_per_step_with_unexpanded_pages():
    method = _Batched()
    runner = _runner(a=_request(blocks=(2, 0)), b=_request(computed=1000, prompt=1044, blocks=(5, 7)),
                     c=_request(max_tokens=8))
    p = BatchedCompressionProvider(method, runner, scheduler_block_size=256)
    plans = {"a": CompressionPlan(300, 128, (2, 0), (50,)), "b": CompressionPlan(1044, 128, (5, 7), (60,)),
             "c": CompressionPlan(300, 128, (2, 0, 3), (70,))}
    spec = MethodRuntimeSpec(True, 256, 128, 128, 64)
    p.runtime_spec = spec
    p.compress_scheduled_requests(_output(plans, {"a": 44, "b": 44, "c": 44}))
    assert len(method.calls) == 1  # c is skipped: its output limit is below the method's minimum
    reqs, kw = method.calls[0]
    assert kw == {"stage_commit": True, "cache_blocks_per_page": 2}
    assert [r.request_id for r in reqs] == ["a", "b"]
    assert [r.source_block_ids_device.tolist() for r in reqs] == [[2, 0], [5, 7]]  # pages, not blocks
    assert [r.destination_block_ids_device.tolist() for r in reqs] == [[50], [60]]
    assert p.pending == {"a": PendingCompression(300, 128, (50,)), "b": PendingCompression(1044, 128, (60,))}
    assert p.last_batch_size == 2


def test_per_request_fallback_expands_scheduler_pages():
    method = _Recording()
    p = BatchedCompressionProvider(method, _runner(r=_request(blocks=(2, 0))), scheduler_block_size=2048)
    p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0), (9,))}, {"r": 44}))
    (req,) = method.requests
    assert req.source_block_ids_device.tolist() == [*range(32, 48), *range(0, 16)]
    assert req.destination_block_ids_device.tolist() == list(range(144, 160))


def test_scheduler_blocks_expand_to_consecutive_kernel_cache_blocks():
    got = expand_scheduler_block_ids((2, 0), 16, torch.device("cpu"))
    assert got.tolist() == [*range(32, 48), *range(0, 16)]
    assert expand_scheduler_block_ids((4, 1), 1, "cpu").tolist() == [4, 1]


def test_prefix_caching_private_destination_and_overlap_rejected():
    method = _Recording()
    p = BatchedCompressionProvider(method, _runner(r=_request()))
    p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0, 3), (100,))}, {"r": 44}))
    assert p.pending["r"] == PendingCompression(300, 128, (100,))
    p = BatchedCompressionProvider(_Recording(), _runner(r=_request()))
    with pytest.raises(RuntimeError, match="private destination"):
        p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0, 3), (3,))}, {"r": 44}))
    with pytest.raises(RuntimeError, match="disagrees"):
        p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0, 4), (50,))}, {"r": 44}))
    with pytest.raises(RuntimeError, match="semantic length"):
        p.compress_scheduled_requests(_output({"r": CompressionPlan(299, 128, (2, 0, 3), (50,))}, {"r": 44}))


def test_requests_without_transaction_or_not_at_prompt_end_are_skipped():
    method = _Recording()
    p = BatchedCompressionProvider(method, _runner(r=_request()))
    p.compress_scheduled_requests(_output({}, {"r": 44}))
    p.compress_scheduled_requests(_output({"r": CompressionPlan(301, 128, (2, 0, 3), (50,))}, {"r": 45 - 1 + 1}))
    assert not p.pending and not method.requests


def test_worker_skips_short_decode_request():
    method = _Recording()
    p = BatchedCompressionProvider(method, _runner(r=_request(max_tokens=32)),
                                   runtime_spec=MethodRuntimeSpec(True, 256, 128, 128, 64))
    p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0, 3), (50,))}, {"r": 44}))
    assert not p.pending and not method.requests


def test_repeated_compression_uses_current_physical_window():
    method = _Recording(per_layer=(("model.layers.0.self_attn", 128),))
    p = BatchedCompressionProvider(method, _runner(r=_request(computed=427, blocks=(5, 9))),
                                   layer_names=("model.layers.0.self_attn",))
    p.active["r"] = ActiveCompression(300, 128, (("model.layers.0.self_attn", 64),))
    p.compress_scheduled_requests(_output({"r": CompressionPlan(428, 128, (5, 9), (50,))}, {"r": 1}))
    (req,) = method.requests
    assert req.physical_num_tokens == 256
    assert req.per_layer_physical_num_tokens == (("model.layers.0.self_attn", 192),)
    assert p.pending["r"] == PendingCompression(428, 128, (50,), (("model.layers.0.self_attn", 128),))


def test_invalid_results_fail_closed():
    class _Bad(_Recording):
        def compress(self, request):
            return CompressionResult(physical_num_tokens=64)

    p = BatchedCompressionProvider(_Bad(), _runner(r=_request()))
    with pytest.raises(RuntimeError, match="unexpected length"):
        p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0, 3), (50,))}, {"r": 44}))
    p = BatchedCompressionProvider(_Recording(per_layer=(("x", 500),)), _runner(r=_request()), layer_names=("x",))
    with pytest.raises(RuntimeError, match="positive and <= group maximum"):
        p.compress_scheduled_requests(_output({"r": CompressionPlan(300, 128, (2, 0, 3), (50,))}, {"r": 44}))


def test_worker_commit_truncates_tables_and_activates_offsets():
    request = _request()
    runner = _runner(r=request, s=_request())
    p = BatchedCompressionProvider(_Recording(), runner)
    p.pending["r"] = PendingCompression(300, 128, (50,))
    p.before_update_states(_output({}, {"s": 1}))  # r not scheduled: no commit yet
    assert "r" in p.pending and "r" not in p.active
    p.before_update_states(_output({}, {"r": 1}))
    assert request.block_ids == ([50],)
    assert runner.input_batch.block_table.added == (([50],), 0)
    assert p.active["r"] == ActiveCompression(300, 128) and not p.pending
    p.after_update_states(None)
    assert p._request_offsets_cpu[:2].tolist() == [172, 0] and p._has_active_rows
    assert p._request_offsets_device[:2].tolist() == [172, 0]


def test_reset_requests_drop_their_state():
    runner = _runner(r=_request())
    p = BatchedCompressionProvider(_Recording(), runner)
    p.pending["r"] = PendingCompression(300, 128, (50,))
    p.active["r"] = ActiveCompression(300, 128)
    out = _output({}, {"r": 1})
    out.preempted_req_ids = {"r"}
    p.before_update_states(out)
    assert not p.pending and not p.active
    p.active["gone"] = ActiveCompression(300, 128)
    p.after_update_states(None)
    assert "gone" not in p.active and not p._has_active_rows


def test_uncompressed_batch_leaves_positions_untouched():
    p = BatchedCompressionProvider(_Recording(), _runner(r=_request()))
    p.after_update_states(None)
    pos = torch.tensor([300, 20])
    assert p.physical_positions_for_slot_mapping(pos) is pos
    p.apply_physical_attention_lengths()  # nothing active: no length change, no device call

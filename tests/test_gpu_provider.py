"""Decode offsets, scheduler-page expansion and the batched provider path on the GPU (through the C ABI).

* ``kvc_decode_offsets`` against the oracle's ``shift_positions`` and
  ``seq_lens - offsets`` on ragged batches (int32/int64 request indices and
  lengths, uncompressed rows at offset 0), the reference provider test's known
  answer, and the range flag for a request index outside the offsets table.
* ``kvc_expand_block_ids`` against the reference's expansion formula.
* ``compress_many`` given 2048-token scheduler pages (16 kernel blocks each, the
  Qwen3.5 layout) equals the same call given expanded kernel-block tables:
  keep indices, compacted bytes, and staged rows that name the pages.
* ``BatchedCompressionProvider`` driving TriAttention for a whole step equals
  the reference's per-request loop (``compress`` per request), then commits
  and shifts the next decode step's positions and lengths.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

import kvc_workloads as W
from oracle import triattention_oracle as O
from vllm_ascend_kvcompress import _native as N
from vllm_ascend_kvcompress.methods.triattention import kernels as K
from vllm_ascend_kvcompress.provider import ActiveCompression, BatchedCompressionProvider
from vllm_ascend_kvcompress.transaction import PLAN_ATTRIBUTE, CompressionPlan

pytestmark = pytest.mark.gpu


def test_decode_offsets_known_answer():
    dev = torch.device("cuda")
    offsets = torch.tensor([172, 0], dtype=torch.int64, device=dev)
    pos = torch.tensor([300, 20], dtype=torch.int64, device=dev)
    out = torch.empty_like(pos)
    K.decode_offsets(offsets, positions=pos, request_indices=torch.tensor([0, 1], device=dev), physical_positions=out)
    lens = torch.tensor([301, 21], dtype=torch.int64, device=dev)
    sem = torch.empty_like(lens)
    K.decode_offsets(offsets, seq_lens=lens, semantic_seq_lens=sem, num_reqs=2)
    assert out.tolist() == [128, 20] and pos.tolist() == [300, 20]
    assert lens.tolist() == [129, 21] and sem.tolist() == [301, 21]


@pytest.mark.parametrize("idx_dtype,len_dtype", [(torch.int32, torch.int32), (torch.int64, torch.int64),
                                                 (torch.int32, torch.int64)])
def test_decode_offsets_match_the_oracle_on_a_ragged_batch(idx_dtype, len_dtype):
    g = torch.Generator().manual_seed(5)
    R = 37
    offsets = torch.randint(0, 50000, (R,), generator=g)
    offsets[::3] = 0  # never-compressed rows
    counts = torch.randint(0, 9, (R,), generator=g)
    req = torch.repeat_interleave(torch.arange(R), counts)
    seq = torch.randint(60000, 120000, (R,), generator=g)
    pos = torch.cat([seq[r] - torch.arange(int(counts[r]), 0, -1) for r in range(R)])
    ref_pos = O.shift_positions(pos, req, offsets)
    dev = torch.device("cuda")
    d_off = offsets.to(dev)
    out = torch.full_like(pos, -1, device=dev)
    lens = seq.to(dev, len_dtype)
    sem = torch.zeros_like(lens)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    K.decode_offsets(d_off, positions=pos.to(dev), request_indices=req.to(dev, idx_dtype), physical_positions=out,
                     error_flag=err)
    K.decode_offsets(d_off, seq_lens=lens, semantic_seq_lens=sem, num_reqs=R - 2, error_flag=err)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), ref_pos)
    assert torch.equal(lens.cpu()[: R - 2].long(), (seq - offsets)[: R - 2])
    assert torch.equal(lens.cpu()[R - 2:].long(), seq[R - 2:])  # rows past num_reqs untouched
    assert torch.equal(sem.cpu()[: R - 2].long(), seq[: R - 2])
    assert int(err.item()) == 0


def test_decode_offsets_flag_an_index_outside_the_table():
    dev = torch.device("cuda")
    offsets = torch.tensor([5, 7], dtype=torch.int64, device=dev)
    pos = torch.tensor([10, 11, 12], dtype=torch.int64, device=dev)
    out = torch.empty_like(pos)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    K.decode_offsets(offsets, positions=pos, request_indices=torch.tensor([0, 2, 1], device=dev),
                     physical_positions=out, error_flag=err)
    torch.cuda.synchronize()
    assert out.tolist() == [5, 11, 5] and int(err.item()) == N.DEV_INDEX_RANGE


@pytest.mark.parametrize("bpp", [1, 9, 16])
def test_expand_block_ids_matches_the_reference_formula(bpp):
    ids = torch.tensor([2, 0, 7, 3], dtype=torch.int64)
    got = K.expand_block_ids(ids.cuda(), bpp).cpu()
    ref = (ids.unsqueeze(1) * bpp + torch.arange(bpp)).reshape(-1)
    assert torch.equal(got, ref)


def _paged_workload() -> W.Workload:
    geo = W.Geometry(2, 2, 16, 256, 64, 1e7, model_type="qwen3_5_moe_text")
    opts = W.Options(kv_budget=4608, recompute_window=1024, protected_prefix_window=128,
                     protected_recent_window=512, score_layer_stride=2)
    return W.place_blocks(W.Workload("paged", geo, opts, [6000, 9000, 12000], seed=21, cache_blocks_per_page=16))


def _caches(w: W.Workload):
    return [tuple(t.cuda() for t in W.kv_pages(w, layer)) for layer in range(w.geometry.num_layers)]


def test_compress_many_takes_scheduler_pages(tmp_path):
    w = _paged_workload()
    a, b = _caches(w), _caches(w)
    ma = W.b200_method(w, a, W.write_stats_file(w, str(tmp_path)))
    mb = W.b200_method(w, b, W.write_stats_file(w, str(tmp_path)))
    ma.compress_many(W.b200_requests(w), stage_commit=True)
    keep_a = ma._keep_view(3).clone()
    mb.compress_many(W.b200_requests(w, pages=True), stage_commit=True, cache_blocks_per_page=16)
    keep_b = mb._keep_view(3).clone()
    ma.check_device_errors()
    mb.check_device_errors()
    assert torch.equal(keep_a, keep_b)
    for (ka, va), (kb, vb) in zip(a, b):
        assert torch.equal(ka.view(torch.int16), kb.view(torch.int16))
        assert torch.equal(va.view(torch.int16), vb.view(torch.int16))
    # staged rows name the scheduler pages; offsets are semantic - budget
    assert mb.staged_block_rows.cpu().tolist() == [w.dst_pages[i] for i in w.compressed()]
    assert ma.staged_block_rows.shape[1] == 36  # kernel blocks without the factor
    assert mb.staged_offsets.cpu().tolist() == [w.lengths[i] - 4608 for i in w.compressed()]


def _runner(w: W.Workload, dev):
    reqs = {}
    for i in w.compressed():
        T = w.lengths[i]
        reqs[f"r{i}"] = SimpleNamespace(num_computed_tokens=T - 7, num_prompt_tokens=T, max_tokens=256,
                                        block_ids=(list(w.src_pages[i]),))
    ids = list(reqs)

    class _Table:
        def add_row(self, block_ids, row):
            self.last = (block_ids, row)

    return SimpleNamespace(device=dev, requests=reqs, max_num_reqs=8, max_num_tokens=64,
                           input_batch=SimpleNamespace(req_ids=ids, num_reqs=len(ids),
                                                       req_id_to_index={r: j for j, r in enumerate(ids)},
                                                       block_table=_Table()),
                           req_indices=SimpleNamespace(gpu=torch.arange(len(ids), dtype=torch.int32, device=dev)),
                           seq_lens=torch.tensor([w.lengths[i] + 1 for i in w.compressed()], dtype=torch.int32,
                                                 device=dev),
                           optimistic_seq_lens_cpu=torch.tensor([w.lengths[i] + 1 for i in w.compressed()],
                                                                dtype=torch.int32))


def test_provider_batches_a_step_like_the_per_request_loop(tmp_path):
    w = _paged_workload()
    dev = torch.device("cuda", 0)
    a, b = _caches(w), _caches(w)
    ma = W.b200_method(w, a, W.write_stats_file(w, str(tmp_path)))
    mb = W.b200_method(w, b, W.write_stats_file(w, str(tmp_path)))
    ra, rb = _runner(w, dev), _runner(w, dev)
    batched = BatchedCompressionProvider(ma, ra, scheduler_block_size=2048)
    per_request = BatchedCompressionProvider(SimpleNamespace(name=mb.name, runtime_spec=mb.runtime_spec,
                                                             compress=mb.compress), rb, scheduler_block_size=2048)
    plans = {f"r{i}": CompressionPlan(w.lengths[i], 4608, tuple(w.src_pages[i]), tuple(w.dst_pages[i]))
             for i in w.compressed()}
    out = SimpleNamespace(num_scheduled_tokens={r: 7 for r in plans}, finished_req_ids=set(),
                          preempted_req_ids=set(), scheduled_cached_reqs=SimpleNamespace(resumed_req_ids=set()))
    setattr(out, PLAN_ATTRIBUTE, plans)
    batched.compress_scheduled_requests(out)
    per_request.compress_scheduled_requests(out)
    ma.check_device_errors()
    mb.check_device_errors()
    assert batched.last_batch_size == 3 and batched.pending == per_request.pending
    for (ka, va), (kb, vb) in zip(a, b):
        assert torch.equal(ka.view(torch.int16), kb.view(torch.int16))
        assert torch.equal(va.view(torch.int16), vb.view(torch.int16))
    # commit on the next step, then the decode step's positions and lengths
    nxt = SimpleNamespace(num_scheduled_tokens={r: 1 for r in plans}, finished_req_ids=set(),
                          preempted_req_ids=set(), scheduled_cached_reqs=SimpleNamespace(resumed_req_ids=set()))
    batched.before_update_states(nxt)
    assert all(ra.requests[r].block_ids == (list(plans[r].destination_block_ids),) for r in plans)
    per_layer = tuple((c.name, 4608) for c in ma.materialization_caches)
    assert batched.active == {f"r{i}": ActiveCompression(w.lengths[i], 4608, per_layer) for i in w.compressed()}
    batched.after_update_states(nxt)
    positions = torch.tensor([w.lengths[i] for i in w.compressed()], dtype=torch.int64, device=dev)
    phys = batched.physical_positions_for_slot_mapping(positions)
    batched.apply_physical_attention_lengths()
    batched.check_device_errors()
    assert phys.tolist() == [4608] * 3 and positions.tolist() == [w.lengths[i] for i in w.compressed()]
    assert ra.seq_lens.tolist() == [4609] * 3 and ra.optimistic_seq_lens_cpu.tolist() == [4609] * 3
    sem_dev, sem_cpu = batched.semantic_seq_lens
    assert sem_dev[:3].tolist() == [w.lengths[i] + 1 for i in w.compressed()]
    assert sem_cpu[:3].tolist() == [w.lengths[i] + 1 for i in w.compressed()]

"""GPU parity of the full score -> select -> compact pass (CUDA path via the C ABI).

Compared with the reference's golden vectors (tests/golden) and with the CPU
oracle on the same seeded inputs: scores within 1e-3 * max(|ref|, 1); kept
indices identical except at near ties (oracle score within that tolerance of
its segment's kept/evicted boundary); compacted K/V bytes identical.
"""

from __future__ import annotations

import hashlib

import pytest
import torch

import kvc_workloads as W
from cases import cpu_caches, golden, golden_small_cases
from gpu_cases import (
    assert_compaction,
    assert_scores_close,
    assert_selection,
    bind,
    oracle_select,
    page_offsets,
    to_gpu,
)

pytestmark = pytest.mark.gpu


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _workload(name: str) -> W.Workload:
    return W.config0() if name == "config0" else golden_small_cases()[name]


@pytest.mark.parametrize("name,scorer", [("config0", "auto"), ("partial", "auto"), ("global_max", "auto"),
                                         ("score_max", "auto"), ("config0", "fma"), ("partial", "fma"),
                                         ("config0", "tcgen05"), ("partial", "tcgen05"),
                                         ("global_max", "tcgen05")])
def test_pipeline_matches_reference_golden(name, scorer, tmp_path, monkeypatch):
    monkeypatch.setenv("KVC_B200_SCORER", scorer)
    arrays, spec = golden()
    w = _workload(name)
    cpu = cpu_caches(w)
    gpu = to_gpu(cpu)
    m = bind(w, gpu, tmp_path)
    if name != "score_max" and scorer == "auto":
        assert m.use_tensor_scorer, "supported geometry must take the tensor-core scorer"
    assert m.use_tcgen05 == (scorer == "tcgen05")
    reqs = W.b200_requests(w)
    idx = w.compressed()
    keep = m.select_many(reqs).cpu()
    raw, mean, var, agg = (t.detach().cpu() for t in m.last_stats)
    offs = page_offsets(w, idx)
    heads = m.local_kv_heads * m.group
    pages = raw.numel() // (m.scoring_layer_count * heads * 128)
    # raw scores are page-major: [layer][page][query head][128 tokens]
    raw = raw.view(m.scoring_layer_count, pages, heads, 128).permute(0, 2, 1, 3).reshape(
        m.scoring_layer_count, heads, pages * 128)
    for row, i in enumerate(idx):
        t = w.lengths[i]
        g_agg = torch.from_numpy(arrays[f"{name}/r{i}/agg"])
        assert_scores_close(agg[offs[row]:offs[row] + t], g_agg)
        g_raw = torch.from_numpy(arrays[f"{name}/r{i}/raw_head"]).reshape(heads, -1)
        assert_scores_close(raw[0, :, offs[row]:offs[row] + g_raw.shape[1]], g_raw)
        R = len(idx)
        mu = mean.view(m.scoring_layer_count, R, heads)[0, row]
        vv = var.view(m.scoring_layer_count, R, heads)[0, row]
        torch.testing.assert_close(mu, torch.from_numpy(arrays[f"{name}/r{i}/mean"]).flatten(), rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(vv, torch.from_numpy(arrays[f"{name}/r{i}/var"]).flatten(), rtol=1e-4, atol=1e-4)
        assert_selection(w, g_agg, torch.from_numpy(arrays[f"{name}/r{i}/keep"]), keep[row])
    m.compress_many(reqs)
    m.check_device_errors()
    torch.cuda.synchronize()
    assert_compaction(w, cpu, gpu, {i: keep[row] for row, i in enumerate(idx)})
    # where the selection is identical, the compacted pages hash like the reference's
    for row, i in enumerate(idx):
        if torch.equal(keep[row], torch.from_numpy(arrays[f"{name}/r{i}/keep"])):
            dst = torch.tensor(w.dst_tables[i])
            for li, (kg, vg) in enumerate(gpu):
                assert _sha(kg[dst.cuda()].cpu()) == spec[name]["dest_hashes"][f"r{i}/layer{li}/k"]
                assert _sha(vg[dst.cuda()].cpu()) == spec[name]["dest_hashes"][f"r{i}/layer{li}/v"]


def test_tensor_and_cuda_core_scorers_agree(tmp_path, monkeypatch):
    w = W.config0()
    gpu = to_gpu(cpu_caches(w))
    out = {}
    for scorer in ("tensor", "tcgen05", "fma"):
        monkeypatch.setenv("KVC_B200_SCORER", scorer)
        m = bind(w, gpu, tmp_path)
        m.select_many(W.b200_requests(w))
        out[scorer] = [t.detach().clone().cpu() for t in m.last_stats]
    for tc in ("tensor", "tcgen05"):
        for a, b in zip(out[tc][1:], out["fma"][1:]):  # mean, var, agg
            finite = torch.isfinite(b)
            assert_scores_close(a[finite], b[finite], tol=2e-4)


def test_per_request_compress_equals_batched(tmp_path):
    w = W.config0()
    cpu = cpu_caches(w)
    g1, g2 = to_gpu(cpu), to_gpu(cpu)
    m1, m2 = bind(w, g1, tmp_path), bind(w, g2, tmp_path)
    reqs1, reqs2 = W.b200_requests(w), W.b200_requests(w)
    for r in reqs1:
        res = m1.compress(r)
        assert res.physical_num_tokens == w.options.kv_budget
    m2.compress_many(reqs2, stage_commit=True)
    torch.cuda.synchronize()
    for (k1, v1), (k2, v2) in zip(g1, g2):
        assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))
        assert torch.equal(v1.view(torch.int16), v2.view(torch.int16))
    rows = m2.staged_block_rows.cpu()
    for row, i in enumerate(w.compressed()):
        assert rows[row].tolist() == w.dst_tables[i][: rows.shape[1]]
        assert int(m2.staged_offsets[row]) == w.lengths[i] - w.options.kv_budget


@pytest.mark.parametrize("scorer", ["tensor", "tcgen05", "fma"])
def test_single_call_step_equals_entry_points_one_by_one(scorer, tmp_path, monkeypatch):
    """kvc_triattention_run launches exactly what the individual entry points do."""
    from vllm_ascend_kvcompress import _native as N
    from vllm_ascend_kvcompress.methods.triattention import kernels as K

    monkeypatch.setenv("KVC_B200_SCORER", scorer)
    w = W.config0()
    cpu = cpu_caches(w)
    g1, g2 = to_gpu(cpu), to_gpu(cpu)
    m = bind(w, g1, tmp_path)
    reqs = W.b200_requests(w)
    m.compress_many(reqs)
    m.check_device_errors()
    keep1 = m._ws.get("keep", len(reqs) * w.options.kv_budget, torch.int64).clone()
    agg1 = m.last_stats[3].clone()
    # the same step through the per-stage entry points, on a second copy of the caches
    m2 = bind(w, g2, tmp_path)
    plan = m2._plan([(r.physical_num_tokens, r.semantic_num_tokens, r.source_block_ids_device,
                      r.destination_block_ids_device) for r in reqs])
    m2._gather_tables(plan)
    L, heads, R, tok = m2.scoring_layer_count, m2.local_kv_heads * m2.group, plan.num_requests, plan.tok_total
    parts = int(N.lib().kvc_tc_partials_per_page()) if m2.use_tensor_scorer else 1
    f32 = lambda n: torch.empty(n, dtype=torch.float32, device="cuda")
    raw, partial = f32(L * heads * tok), f32(L * plan.total_pages * parts * heads * 2)
    mean, var, den, rows, agg = f32(L * R * heads), f32(L * R * heads), f32(L * R * heads), f32(L * tok), f32(tok)
    keep = torch.empty(R * w.options.kv_budget, dtype=torch.int64, device="cuda")
    if m2.use_tensor_scorer:
        frag = torch.empty(R * L * m2.local_kv_heads * m2.frag_block, dtype=torch.int32, device="cuda")
        K.prepare_score_fragments(m2.scoring_omega, m2.offsets, plan, m2.scoring_q_real, m2.scoring_q_imag,
                                  m2.scoring_scale, m2.scoring_extra, m2.scoring_q_pass, m2.kv_dtype, frag,
                                  tcgen05=m2.use_tcgen05)
        K.score_paged_keys_tc(m2._key_maps, L, m2.kv_dtype, m2.num_blocks, m2.local_kv_heads, m2.group,
                              m2.head_dim, m2.rotary_dim, plan, frag, raw, partial, m2._err, tcgen05=m2.use_tcgen05)
    else:
        coef = f32(R * L * m2.local_kv_heads * m2.coef_block)
        K.prepare_score_coefficients(m2.scoring_omega, m2.offsets, plan, m2.scoring_q_real, m2.scoring_q_imag,
                                     m2.scoring_scale, m2.scoring_extra, m2.score_aggregation_code, coef)
        K.score_paged_keys(m2._k_score, m2.kv_dtype, m2.block_stride, m2.num_blocks, m2.local_kv_heads, m2.group,
                           m2.head_dim, m2.rotary_dim, plan, coef, m2.offsets.numel(), m2.score_aggregation_code,
                           m2.scoring_q_pass_t, raw, partial, m2._err)
    K.head_stats(partial, L, heads, plan, mean, var, den, parts)
    K.normalize_aggregate(raw, L, heads, plan, mean, den, m2.layer_aggregation_code, rows_out=rows, agg_out=agg)
    cfg = m2.config
    K.select_keep(agg, plan, cfg.kv_budget, cfg.protected_prefix_window, cfg.protected_recent_window,
                  cfg.position_segments, N.POLICY_V3, keep, m2._err)
    K.compact(m2._k_all, m2._v_all, m2.block_stride_bytes, m2.num_blocks, m2.row_bytes, plan, keep,
              cfg.kv_budget, m2._err, None, None)
    torch.cuda.synchronize()
    assert int(m2._err.item()) == 0
    assert torch.equal(agg.view(torch.int32), agg1.view(torch.int32))
    assert torch.equal(keep, keep1)
    for (k1, v1), (k2, v2) in zip(g1, g2):
        assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))
        assert torch.equal(v1.view(torch.int16), v2.view(torch.int16))


def test_block_tables_of_any_int_dtype_and_padding_give_the_same_step(tmp_path):
    """Tables longer than needed, int32, or strided views are gathered like exact int64 tables."""
    from dataclasses import replace

    w = W.config0()
    cpu = cpu_caches(w)
    g1, g2 = to_gpu(cpu), to_gpu(cpu)
    m1, m2 = bind(w, g1, tmp_path), bind(w, g2, tmp_path)
    reqs = W.b200_requests(w)
    m1.compress_many(reqs)
    odd = []
    for j, r in enumerate(reqs):
        src = torch.cat([r.source_block_ids_device, torch.full((5,), -7, device="cuda", dtype=torch.int64)])
        dst = torch.stack([r.destination_block_ids_device, r.destination_block_ids_device], 1)[:, 0]  # strided
        odd.append(replace(r, source_block_ids_device=src.to(torch.int32) if j % 2 else src,
                           destination_block_ids_device=dst))
    m2.compress_many(odd)
    m1.check_device_errors()
    m2.check_device_errors()
    torch.cuda.synchronize()
    for (k1, v1), (k2, v2) in zip(g1, g2):
        assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))
        assert torch.equal(v1.view(torch.int16), v2.view(torch.int16))


def test_later_round_uses_semantic_length_for_phases(tmp_path):
    """A request compressed before has semantic > physical tokens: phases use the semantic count."""
    from dataclasses import replace

    from oracle import triattention_oracle as O
    from cases import oracle_options, oracle_stats

    w = W.config0()
    cpu = cpu_caches(w)
    gpu = to_gpu(cpu)
    m = bind(w, gpu, tmp_path)
    idx = w.compressed()
    extra = [7777, 20000, 123]
    reqs = [replace(r, semantic_num_tokens=r.physical_num_tokens + e) for r, e in zip(W.b200_requests(w), extra)]
    keep = m.select_many(reqs).cpu()
    agg = m.last_stats[3].cpu()
    offs = page_offsets(w, idx)
    stats, opts = oracle_stats(w), oracle_options(w)
    offsets = O.geometric_offsets(w.options.max_model_len)
    for row, (i, e) in enumerate(zip(idx, extra)):
        req = O.OracleRequest(semantic_num_tokens=w.lengths[i] + e, physical_num_tokens=w.lengths[i],
                              src_blocks=torch.tensor(w.src_tables[i]), dst_blocks=torch.tensor(w.dst_tables[i]))
        r_agg, r_keep = O.select_request([c[0] for c in cpu], stats, req, opts, offsets, 1)
        assert_scores_close(agg[offs[row]:offs[row] + w.lengths[i]], r_agg)
        assert_selection(w, r_agg, r_keep, keep[row])
    m.compress_many(reqs, stage_commit=True)
    m.check_device_errors()
    assert m.staged_offsets.cpu().tolist() == [w.lengths[i] + e - w.options.kv_budget for i, e in zip(idx, extra)]


def test_tp4_rows_max_equals_tp1_emulated(tmp_path):
    """Four TP ranks on one GPU: the elementwise max of their rows reproduces TP=1's selection."""
    w = EDGE_CASES["ragged"]
    idx = [i for i, t in enumerate(w.lengths) if t >= w.options.kv_budget]
    cpu = cpu_caches(w)
    full = bind(w, to_gpu(cpu), tmp_path)
    reqs = W.b200_requests(w, indices=idx)
    keep1 = full.select_many(reqs).cpu()
    per = w.geometry.num_kv_heads // 4
    ranks, rows = [], []
    for r in range(4):
        shard = [(k[:, :, r * per:(r + 1) * per].contiguous().cuda(), v[:, :, r * per:(r + 1) * per].contiguous().cuda())
                 for k, v in cpu]
        m = bind(w, shard, tmp_path, tp_size=4, tp_rank=r)
        m._tp_all_reduce_max = lambda x: rows.append(x.clone())
        m.select_many(reqs)
        ranks.append(m)
    best = torch.stack(rows).amax(0)
    for m in ranks:
        m._tp_all_reduce_max = lambda x, b=best: x.copy_(b)
        assert torch.equal(m.select_many(reqs).cpu(), keep1)


def test_select_keep_indices_hook_matches_batch(tmp_path):
    w = W.config0()
    gpu = to_gpu(cpu_caches(w))
    m = bind(w, gpu, tmp_path)
    reqs = W.b200_requests(w)
    batched = m.select_many(reqs).cpu()
    for row, r in enumerate(reqs):
        one = m._select_keep_indices(r.source_block_ids_device, r.physical_num_tokens, r.semantic_num_tokens)
        assert torch.equal(one.cpu(), batched[row])


def test_tp2_rows_and_selection_emulated(tmp_path):
    """Two TP ranks on one GPU; the MAX all-reduce is emulated by exchanging rows."""
    arrays, _ = golden()
    w = golden_small_cases()["partial"]
    cpu = cpu_caches(w)
    half = w.geometry.num_kv_heads // 2
    ranks = []
    for r in (0, 1):
        shard = [(k[:, :, r * half:(r + 1) * half].contiguous().cuda(), v[:, :, r * half:(r + 1) * half].contiguous().cuda())
                 for k, v in cpu]
        ranks.append(bind(w, shard, tmp_path, tp_size=2, tp_rank=r))
    captured = {}
    for r, m in enumerate(ranks):
        def capture(rows, r=r):
            captured[r] = rows.clone()
        m._tp_all_reduce_max = capture
        m.select_many(W.b200_requests(w))
    keeps = []
    for r, m in enumerate(ranks):
        other = captured[1 - r]
        m._tp_all_reduce_max = lambda rows, o=other: torch.maximum(rows, o, out=rows)
        keeps.append(m.select_many(W.b200_requests(w)).cpu())
    assert torch.equal(keeps[0], keeps[1])
    idx = w.compressed()
    offs = page_offsets(w, idx)
    L = ranks[0].scoring_layer_count
    for r in (0, 1):
        rows = captured[r].cpu().view(L, -1)
        for row, i in enumerate(idx):
            t = w.lengths[i]
            assert_scores_close(rows[:, offs[row]:offs[row] + t], torch.from_numpy(arrays[f"partial/r{i}/rows_rank{r}"]))
    for row, i in enumerate(idx):
        assert_selection(w, torch.from_numpy(arrays[f"partial/r{i}/agg_tp2"]),
                         torch.from_numpy(arrays[f"partial/r{i}/keep_tp2"]), keeps[0][row])


def _edge(name, geo, opts, lengths, seed, per=1):
    return W.place_blocks(W.Workload(name, geo, opts, lengths, seed=seed, cache_blocks_per_page=per))


EDGE_CASES = {
    # T == budget (nothing evicted), T == budget + 1, lengths off the page grid
    "exact_budget": _edge("exact_budget", W.Geometry(2, 2, 8, 128, 128, 1e6),
                          W.Options(kv_budget=1024, protected_prefix_window=16, protected_recent_window=128,
                                    score_layer_stride=1), [1024, 1025, 1333], 21),
    # more segments than middle tokens -> empty segments
    "many_segments": _edge("many_segments", W.Geometry(1, 1, 4, 64, 64, 1e4),
                           W.Options(kv_budget=256, protected_prefix_window=100, protected_recent_window=140,
                                     position_segments=64, score_layer_stride=1), [300, 420], 22),
    # single query head per KV head, large group, max layer aggregation, global policy
    "g1_global": _edge("g1_global", W.Geometry(3, 4, 4, 128, 128, 1e6),
                       W.Options(kv_budget=512, protected_prefix_window=0, protected_recent_window=0,
                                 position_policy="global", layer_aggregation="max", score_layer_stride=2),
                       [700, 2000, 513], 23),
    "g8_partial": _edge("g8_partial", W.Geometry(2, 1, 8, 256, 64, 1e7, model_type="qwen3_5_moe_text"),
                        W.Options(kv_budget=768, protected_prefix_window=128, protected_recent_window=128,
                                  score_layer_stride=1), [2100, 900], 24, per=16),
    "g2_d64": _edge("g2_d64", W.Geometry(2, 2, 4, 64, 64, 1e4),
                    W.Options(kv_budget=384, protected_prefix_window=8, protected_recent_window=64,
                              position_segments=3, score_layer_stride=1), [1000, 385, 4000], 25),
    # three KV heads of 64 dims: 384-byte rows, not a power-of-two count of vectors
    "kvh3_d64": _edge("kvh3_d64", W.Geometry(2, 3, 6, 64, 64, 1e4),
                      W.Options(kv_budget=512, protected_prefix_window=16, protected_recent_window=64,
                                score_layer_stride=1), [1500, 700, 2600], 27),
    # the longest sequence max_model_len allows: phases at ~2^17 radians, position 65535
    "max_len_64k": _edge("max_len_64k", W.Geometry(1, 2, 4, 128, 128, 1e6),
                         W.Options(kv_budget=4096, protected_prefix_window=128, protected_recent_window=512,
                                   score_layer_stride=1), [65536], 28),
    # a layer count that the stride does not divide: scoring layers 0, 3, 6
    "stride3_7layers": _edge("stride3_7layers", W.Geometry(7, 2, 4, 64, 64, 1e4),
                             W.Options(kv_budget=512, protected_prefix_window=16, protected_recent_window=64,
                                       score_layer_stride=3), [1300, 900, 2100], 29),
    # forty requests in one step
    "forty_requests": _edge("forty_requests", W.Geometry(1, 2, 8, 128, 128, 1e6),
                            W.Options(kv_budget=1024, protected_prefix_window=0, protected_recent_window=128,
                                      score_layer_stride=1),
                            [1024 + (i * 977) % 2000 for i in range(40)], 30),
    # a ragged batch of many requests
    "ragged": _edge("ragged", W.Geometry(2, 8, 40, 128, 128, 1e6),
                    W.Options(kv_budget=640, protected_prefix_window=64, protected_recent_window=128,
                              score_layer_stride=1),
                    [640, 700, 1500, 2049, 3000, 777, 5000, 641, 1280, 4097], 26),
}


@pytest.mark.parametrize("case", sorted(EDGE_CASES))
def test_edge_cases_match_oracle(case, tmp_path):
    w = EDGE_CASES[case]
    idx = [i for i, t in enumerate(w.lengths) if t >= w.options.kv_budget]
    w.dst_tables = [w.dst_tables[i] if w.dst_tables[i] else [] for i in range(len(w.lengths))]
    # method-level: every sequence with T >= budget is compressed (the provider's
    # recompute threshold is a scheduler gate); give each one a destination
    nxt = w.num_blocks
    need = -(-w.options.kv_budget // 128)
    for i in idx:
        if not w.dst_tables[i]:
            w.dst_tables[i] = list(range(nxt, nxt + need))
            nxt += need
    w.num_blocks = nxt
    cpu = cpu_caches(w)
    gpu = to_gpu(cpu)
    m = bind(w, gpu, tmp_path)
    reqs = W.b200_requests(w, indices=idx)
    keep = m.select_many(reqs).cpu()
    agg = m.last_stats[3].cpu()
    ref = oracle_select(w, cpu, idx)
    offs = page_offsets(w, idx)
    for row, i in enumerate(idx):
        r_agg, r_keep = ref[i]
        assert_scores_close(agg[offs[row]:offs[row] + w.lengths[i]], r_agg)
        assert_selection(w, r_agg, r_keep, keep[row])
    m.compress_many(reqs)
    m.check_device_errors()
    torch.cuda.synchronize()
    assert_compaction(w, cpu, gpu, {i: keep[row] for row, i in enumerate(idx)})


@pytest.mark.parametrize("scorer", ["auto", "tcgen05"])
def test_fp16_cache_and_padded_block_stride(scorer, tmp_path, monkeypatch):
    """K and V interleaved in one raw buffer with padding between pages, fp16."""
    monkeypatch.setenv("KVC_B200_SCORER", scorer)
    w = _edge("padded_fp16", W.Geometry(2, 2, 10, 128, 128, 1e6),
              W.Options(kv_budget=512, protected_prefix_window=4, protected_recent_window=64, score_layer_stride=1),
              [900, 1700], 27)
    page = 128 * 2 * 128
    stride = 2 * page + 64
    cpu, gpu = [], []
    for layer in range(2):
        k, v = W.kv_pages(w, layer, dtype=torch.float16)
        raw = torch.full((w.num_blocks * stride,), -7.0, dtype=torch.float16)
        kv = torch.as_strided(raw, k.shape, (stride, 256, 128, 1))
        vv = torch.as_strided(raw, k.shape, (stride, 256, 128, 1), storage_offset=page)
        kv.copy_(k)
        vv.copy_(v)
        cpu.append((kv, vv, raw))
        graw = raw.cuda()
        gpu.append((torch.as_strided(graw, k.shape, (stride, 256, 128, 1)),
                    torch.as_strided(graw, k.shape, (stride, 256, 128, 1), storage_offset=page), graw))
    m = bind(w, [(a, b) for a, b, _ in gpu], tmp_path)
    idx = w.compressed()
    reqs = W.b200_requests(w, indices=idx)
    keep = m.select_many(reqs).cpu()
    ref = oracle_select(w, [(a, b) for a, b, _ in cpu], idx)
    for row, i in enumerate(idx):
        assert_selection(w, ref[i][0], ref[i][1], keep[row])
    m.compress_many(reqs)
    torch.cuda.synchronize()
    assert_compaction(w, [(a, b) for a, b, _ in cpu], [(a, b) for a, b, _ in gpu],
                      {i: keep[row] for row, i in enumerate(idx)})
    for (_, _, raw), (_, _, graw) in zip(cpu, gpu):
        pad = graw.view(w.num_blocks, stride)[:, -64:].cpu()
        assert bool((pad == -7.0).all()), "padding between pages must stay untouched"


@pytest.mark.parametrize("scorer", ["auto", "tcgen05"])
def test_fp16_partial_rope_matches_oracle(scorer, tmp_path, monkeypatch):
    """FP16 caches with partial RoPE (head_dim 256, rotary 64, 8 query heads per KV head)."""
    monkeypatch.setenv("KVC_B200_SCORER", scorer)
    w = _edge("fp16_partial", W.Geometry(2, 1, 8, 256, 64, 1e7, model_type="qwen3_5_moe_text"),
              W.Options(kv_budget=768, protected_prefix_window=128, protected_recent_window=128,
                        score_layer_stride=1), [2100, 1500], 31, per=16)
    cpu = [W.kv_pages(w, layer, dtype=torch.float16) for layer in range(w.geometry.num_layers)]
    gpu = to_gpu(cpu)
    m = bind(w, gpu, tmp_path)
    assert m.use_tensor_scorer and m.kv_dtype == torch.float16
    idx = w.compressed()
    reqs = W.b200_requests(w, indices=idx)
    keep = m.select_many(reqs).cpu()
    agg = m.last_stats[3].cpu()
    ref = oracle_select(w, cpu, idx)
    offs = page_offsets(w, idx)
    for row, i in enumerate(idx):
        assert_scores_close(agg[offs[row]:offs[row] + w.lengths[i]], ref[i][0])
        assert_selection(w, ref[i][0], ref[i][1], keep[row])
    m.compress_many(reqs)
    m.check_device_errors()
    torch.cuda.synchronize()
    assert_compaction(w, cpu, gpu, {i: keep[row] for row, i in enumerate(idx)})


def test_device_range_errors_are_reported(tmp_path):
    w = W.config0()
    gpu = to_gpu(cpu_caches(w))
    m = bind(w, gpu, tmp_path)
    reqs = W.b200_requests(w)
    bad = reqs[0].source_block_ids_device.clone()
    bad[3] = 10_000_000
    from dataclasses import replace

    m.compress_many([replace(reqs[0], source_block_ids_device=bad)])
    with pytest.raises(RuntimeError, match="block id outside"):
        m.check_device_errors()
    m.compress_many(reqs)  # the flag was cleared; a good batch passes
    m.check_device_errors()


def test_host_validation_fails_closed(tmp_path):
    w = W.config0()
    gpu = to_gpu(cpu_caches(w))
    m = bind(w, gpu, tmp_path)
    reqs = W.b200_requests(w)
    from dataclasses import replace

    with pytest.raises(ValueError, match="budget"):
        m.compress(replace(reqs[0], physical_num_tokens=1000))
    with pytest.raises(RuntimeError, match="destination"):
        m.compress(replace(reqs[0], destination_block_ids_device=reqs[0].destination_block_ids_device[:3]))
    with pytest.raises(RuntimeError, match="source block table"):
        m.compress(replace(reqs[0], source_block_ids_device=reqs[0].source_block_ids_device[:2]))

"""Generate golden vectors by running the REFERENCE plugin on seeded CPU inputs.

Usage (in a container that has the reference checkout)::

    KVC_REFERENCE_SRC=/path/to/vllm-ascend-kvcompress-hust/src \
        python tests/golden/make_golden.py

The reference package (``vllm_ascend_kvcompress`` 0.10.0) is imported from
``KVC_REFERENCE_SRC``; on a non-NPU device its TriAttention method runs its
torch fallback path, which is the behaviour these fixtures record.  Inputs are
rebuilt deterministically by ``kvc_workloads`` from the seeds stored beside the
outputs, so only outputs (and small raw-score excerpts) are committed.

Outputs: ``tests/golden/golden.npz`` plus ``tests/golden/golden.json`` (case
specs and hashes of compacted pages).  This script never runs on the GPU box.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if not os.environ.get("KVC_REFERENCE_SRC"):
    raise SystemExit("set KVC_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, os.environ["KVC_REFERENCE_SRC"])
sys.path.insert(1, str(ROOT))

import kvc_workloads as W  # noqa: E402
import vllm_ascend_kvcompress.calibration as ref_calib  # noqa: E402
import vllm_ascend_kvcompress.methods.triattention.method as ref_method  # noqa: E402
from vllm_ascend_kvcompress.methods.base import (  # noqa: E402
    CompressionRequest,
    LayerCache,
    ModelShape,
)

torch.set_num_threads(min(8, os.cpu_count() or 1))


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def model_shape(geo: W.Geometry) -> ModelShape:
    return ModelShape(
        model_type=geo.model_type,
        num_layers=geo.num_layers,
        num_attention_heads=geo.num_q_heads,
        num_kv_heads=geo.num_kv_heads,
        head_dim=geo.head_dim,
        rope_theta=geo.rope_theta,
        has_rope_scaling=False,
        rotary_dim=None if geo.rotary_dim == geo.head_dim else geo.rotary_dim,
    )


def bind(w: W.Workload, caches, stats_path: str, tp_size: int = 1, tp_rank: int = 0):
    vcfg = SimpleNamespace(
        parallel_config=SimpleNamespace(tensor_parallel_size=tp_size),
        model_config=SimpleNamespace(max_model_len=w.options.max_model_len),
        speculative_config=None,
    )
    m = ref_method.TriAttentionMethod(w.options.method_config(stats_path), vcfg, model_shape(w.geometry))
    layers = tuple(
        LayerCache(name=f"model.layers.{i}.self_attn.attn", layer_index=i, k_cache=k, v_cache=v)
        for i, (k, v) in enumerate(caches)
    )
    if tp_size > 1:
        import vllm.distributed as vd

        orig = vd.get_tp_group
        vd.get_tp_group = lambda: SimpleNamespace(rank_in_group=tp_rank, device_group="tp")
        try:
            m.bind_model_runner(SimpleNamespace(device=torch.device("cpu")), layers)
        finally:
            vd.get_tp_group = orig
    else:
        m.bind_model_runner(SimpleNamespace(device=torch.device("cpu")), layers)
    return m


def write_stats(w: W.Workload, tmp: Path) -> str:
    path = tmp / f"{w.name}-stats.pt"
    torch.save(W.calibration_payload(w.geometry, w.seed), path)
    return str(path)


def request(w: W.Workload, i: int) -> CompressionRequest:
    src = torch.tensor(w.src_tables[i], dtype=torch.long)
    dst = torch.tensor(w.dst_tables[i], dtype=torch.long)
    return CompressionRequest(
        request_id=f"r{i}",
        semantic_num_tokens=w.lengths[i],
        physical_num_tokens=w.lengths[i],
        source_block_ids=(tuple(w.src_tables[i]),),
        destination_block_ids=(tuple(w.dst_tables[i]),),
        source_block_ids_device=src,
        destination_block_ids_device=dst,
    )


def run_case(w: W.Workload, tmp: Path, arrays: dict, spec: dict, raw_excerpt: int = 256) -> None:
    caches = [W.kv_pages(w, layer) for layer in range(w.geometry.num_layers)]
    stats_path = write_stats(w, tmp)
    m = bind(w, caches, stats_path)
    hashes = {}
    for i in w.compressed():
        req = request(w, i)
        t = w.lengths[i]
        keep = m._select_keep_indices(req.source_block_ids_device, t, t)
        arrays[f"{w.name}/r{i}/agg"] = m.aggregate_workspace[:t].clone().numpy()
        arrays[f"{w.name}/r{i}/keep"] = keep.numpy().astype(np.int64)
        # raw per-head scores of the first scoring layer, recomputed by the
        # reference scorer itself on the gathered keys
        layer0 = m.layer_caches[0]
        keys = ref_method.gather_paged_range(
            layer0.k_cache, req.source_block_ids_device, start=0, count=t, block_size=128
        )
        raw = ref_method.score_post_rope_keys(
            keys, layer0.stats, round_start=t, offsets=m.offsets,
            aggregation=w.options.score_aggregation,
        )
        var, mean = torch.var_mean(raw, dim=-1, correction=0)
        arrays[f"{w.name}/r{i}/raw_head"] = raw[..., :raw_excerpt].clone().numpy()
        arrays[f"{w.name}/r{i}/mean"] = mean.numpy()
        arrays[f"{w.name}/r{i}/var"] = var.numpy()
        m.compress(req)
        for li, (k, v) in enumerate(caches):
            dst = torch.tensor(w.dst_tables[i])
            hashes[f"r{i}/layer{li}/k"] = sha(k[dst])
            hashes[f"r{i}/layer{li}/v"] = sha(v[dst])
    spec[w.name] = {
        "lengths": w.lengths,
        "seed": w.seed,
        "compressed": w.compressed(),
        "dest_hashes": hashes,
    }


def run_tp2(w: W.Workload, tmp: Path, arrays: dict, spec: dict) -> None:
    """TP=2: each rank holds one half of the KV heads; rows are MAX-reduced."""
    import torch.distributed as dist

    caches = [W.kv_pages(w, layer) for layer in range(w.geometry.num_layers)]
    stats_path = write_stats(w, tmp)
    half = w.geometry.num_kv_heads // 2
    shard = lambda r: [(k[:, :, r * half:(r + 1) * half].contiguous(),
                        v[:, :, r * half:(r + 1) * half].contiguous()) for k, v in caches]
    ranks = [bind(w, shard(r), stats_path, tp_size=2, tp_rank=r) for r in (0, 1)]
    import vllm.distributed as vd

    orig_ar, orig_g = dist.all_reduce, vd.get_tp_group
    vd.get_tp_group = lambda: SimpleNamespace(rank_in_group=0, device_group="tp")
    try:
        for i in w.compressed():
            t = w.lengths[i]
            req = request(w, i)
            rows = {}

            def capture(rank):
                def fake(scores, *, op, group):
                    assert op == dist.ReduceOp.MAX
                    rows[rank] = scores.clone()
                return fake

            for r in (0, 1):
                dist.all_reduce = capture(r)
                ranks[r]._select_keep_indices(req.source_block_ids_device, t, t)
            keeps = []
            for r in (0, 1):
                other = rows[1 - r]
                dist.all_reduce = lambda s, *, op, group, o=other: torch.maximum(s, o, out=s)
                keeps.append(ranks[r]._select_keep_indices(req.source_block_ids_device, t, t))
            assert torch.equal(keeps[0], keeps[1])
            arrays[f"{w.name}/r{i}/rows_rank0"] = rows[0].numpy()
            arrays[f"{w.name}/r{i}/rows_rank1"] = rows[1].numpy()
            arrays[f"{w.name}/r{i}/keep_tp2"] = keeps[0].numpy().astype(np.int64)
            arrays[f"{w.name}/r{i}/agg_tp2"] = ranks[0].aggregate_workspace[:t].clone().numpy()
    finally:
        dist.all_reduce, vd.get_tp_group = orig_ar, orig_g
    spec[w.name + "_tp2"] = {"lengths": w.lengths, "seed": w.seed, "compressed": w.compressed()}


def small_cases() -> list[W.Workload]:
    partial = W.place_blocks(W.Workload(
        "partial", W.Geometry(4, 2, 16, 256, 64, 1e7, model_type="qwen3_5_moe_text"),
        W.Options(kv_budget=1024, recompute_window=128, protected_prefix_window=16,
                  protected_recent_window=128, score_layer_stride=2, score_chunk_size=512),
        [1400, 2000], seed=5, cache_blocks_per_page=2))
    glob = W.place_blocks(W.Workload(
        "global_max", W.Geometry(3, 2, 4, 64, 64, 1e4),
        W.Options(kv_budget=512, protected_prefix_window=0, protected_recent_window=128,
                  position_policy="global", layer_aggregation="max", score_chunk_size=256,
                  score_layer_stride=1),
        [700, 1000], seed=6))
    maxagg = W.place_blocks(W.Workload(
        "score_max", W.Geometry(2, 1, 4, 64, 64, 1e6),
        W.Options(kv_budget=256, protected_prefix_window=8, protected_recent_window=128,
                  score_aggregation="max", score_layer_stride=1, score_chunk_size=256),
        [600], seed=7))
    return [partial, glob, maxagg]


def calibration_case(arrays: dict, spec: dict) -> None:
    for name, heads, hd, rot, calls in W.golden_calibration_inputs():
        acc = ref_calib._LayerAccumulator()
        for q in calls:
            acc.add(q, heads, hd, rot)
        arrays[f"{name}/real_sum"] = acc.real_sum.numpy()
        arrays[f"{name}/imag_sum"] = acc.imag_sum.numpy()
        arrays[f"{name}/abs_sum"] = acc.abs_sum.numpy()
        if acc.pass_sum is not None:
            arrays[f"{name}/pass_sum"] = acc.pass_sum.numpy()
        spec[name] = {"heads": heads, "head_dim": hd, "rotary_dim": rot,
                      "calls": [int(q.shape[0]) for q in calls], "count": acc.count}


SELECTION_CASES = [
    # (tokens, budget, prefix, recent, segments, policy) -- the reference's own
    # test_batched_v3_matches_per_segment_selection parameters plus edge shapes
    (32768, 8192, 128, 512, 8, "v3"),
    (32768, 8192, 256, 512, 8, "v3"),
    (32, 17, 0, 0, 4, "v3"),
    (32, 18, 2, 2, 4, "v3"),
    (32, 31, 0, 0, 4, "v3"),
    (19, 13, 2, 2, 8, "v3"),
    (6000, 2048, 4, 128, 8, "v3"),
    (5000, 4608, 128, 512, 8, "v3"),
    (4736, 4608, 128, 512, 8, "v3"),
    (65536, 4608, 128, 512, 8, "v3"),
    (1000, 999, 0, 0, 3, "v3"),
    (3000, 1000, 0, 128, 1, "v3"),
    (3000, 1000, 0, 128, 8, "global"),
    (700, 512, 5, 7, 8, "global"),
]


def selection_cases(arrays: dict, spec: dict) -> None:
    from vllm_ascend_kvcompress.methods.triattention.selection import select_keep_indices

    spec["selection"] = []
    all_scores = W.golden_selection_scores(SELECTION_CASES)
    for n, (t, b, p, r, s, pol) in enumerate(SELECTION_CASES):
        scores = all_scores[n]
        keep = select_keep_indices(scores, budget=b, protected_prefix=p, protected_recent=r,
                                   segments=s, policy=pol)
        arrays[f"selection/{n}/keep"] = keep.numpy().astype(np.int32)
        spec["selection"].append([t, b, p, r, s, pol])


def main() -> None:
    arrays: dict = {}
    spec: dict = {"reference": "vllm-ascend-kvcompress-hust 0.10.0 (torch CPU fallback path)",
                  "torch": torch.__version__}
    with tempfile.TemporaryDirectory() as td:
        tmp = Path(td)
        run_case(W.config0(), tmp, arrays, spec)
        cases = small_cases()
        for w in cases:
            run_case(w, tmp, arrays, spec)
        run_tp2(cases[0], tmp, arrays, spec)
    calibration_case(arrays, spec)
    selection_cases(arrays, spec)
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(spec, indent=1, sort_keys=True) + "\n")
    print("wrote", len(arrays), "arrays")


if __name__ == "__main__":
    main()

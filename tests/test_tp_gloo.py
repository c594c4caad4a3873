"""Tensor-parallel score sync with two real processes (gloo on CPU).

Each rank scores its half of the KV heads with the CPU oracle, then calls the
product's ``tp_score_sync`` (one MAX all-reduce of all per-layer rows of all
requests).  Both ranks must end with identical rows equal to the TP=1 rows, so
their selections agree with each other and with TP=1.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    for p in (str(ROOT), str(ROOT / "vllm-ascend-kvcompress-hust_b200"), str(ROOT / "tests")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import cases
        from oracle import triattention_oracle as O
        from vllm_ascend_kvcompress.methods.triattention.method import tp_score_sync

        w = cases.golden_small_cases()["partial"]
        caches = cases.cpu_caches(w)
        stats = cases.oracle_stats(w)
        opts = cases.oracle_options(w)
        offs = O.geometric_offsets(w.options.max_model_len)
        half = w.geometry.num_kv_heads // world
        rows = []
        for i in w.compressed():
            req = cases.oracle_request(w, i)
            kc = [c[0][:, :, rank * half:(rank + 1) * half] for c in caches]
            rows.append(O.layer_rows(kc, [s.shard(rank, world) for s in stats], req, opts, offs))
        batched = torch.cat([r for r in rows], dim=1).contiguous()  # [L_s, sum T]: one collective per step
        tp_score_sync(batched, dist.group.WORLD)
        torch.save(batched, Path(out_dir) / f"rows{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_tp_score_sync_two_ranks(tmp_path):
    import cases
    from oracle import triattention_oracle as O

    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    r0 = torch.load(tmp_path / "rows0.pt")
    r1 = torch.load(tmp_path / "rows1.pt")
    assert torch.equal(r0, r1)
    w = cases.golden_small_cases()["partial"]
    caches = cases.cpu_caches(w)
    stats = cases.oracle_stats(w)
    opts = cases.oracle_options(w)
    offs = O.geometric_offsets(w.options.max_model_len)
    full = torch.cat([O.layer_rows([c[0] for c in caches], stats, cases.oracle_request(w, i), opts, offs)
                      for i in w.compressed()], dim=1)
    assert torch.equal(r0, full)
    arrays, _ = cases.golden()
    pos = 0
    for i in w.compressed():
        t = w.lengths[i]
        agg = O.aggregate_rows(r0[:, pos:pos + t].contiguous(), opts.layer_aggregation)
        keep = O.select_keep_indices(agg, budget=opts.kv_budget, protected_prefix=opts.protected_prefix_window,
                                     protected_recent=opts.protected_recent_window,
                                     segments=opts.position_segments, policy=opts.position_policy)
        assert keep.tolist() == arrays[f"partial/r{i}/keep_tp2"].tolist()
        pos += t

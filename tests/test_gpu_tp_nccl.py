"""Tensor-parallel score sync on two GPUs (skipped with fewer).

Rank r binds the method to its half of the KV heads.  The per-layer rows are
synchronised either by one NCCL MAX all-reduce per step ("nccl") or by the
peer-memory exchange kernel over NVLink ("peer").  Both ranks must keep the
same indices as a TP=1 run, each rank's compacted local heads must equal the
matching head slice of the TP=1 compaction, and both paths must give the same
scores bit for bit.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
import tempfile
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _workload():
    import kvc_workloads as W

    return W.place_blocks(W.Workload(
        "tp_nccl", W.Geometry(3, 4, 20, 128, 128, 1e6),
        W.Options(kv_budget=1024, protected_prefix_window=32, protected_recent_window=128, score_layer_stride=2),
        [1500, 3100, 2222, 1160], seed=31))


def _rank(rank: int, world: int, port: int, out: str, mode: str) -> None:
    for p in (str(ROOT), str(ROOT / "vllm-ascend-kvcompress-hust_b200"), str(ROOT / "tests")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", KVC_B200_TP_SYNC=mode)
    import torch.distributed as dist

    import kvc_workloads as W

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        w = _workload()
        per = w.geometry.num_kv_heads // world
        caches = []
        for layer in range(w.geometry.num_layers):
            k, v = W.kv_pages(w, layer)
            caches.append((k[:, :, rank * per:(rank + 1) * per].contiguous().to(dev),
                           v[:, :, rank * per:(rank + 1) * per].contiguous().to(dev)))
        with tempfile.TemporaryDirectory() as d:
            m = W.b200_method(w, caches, W.write_stats_file(w, d), tp_size=world, tp_group=dist.group.WORLD,
                              tp_rank=rank, device=dev)
        reqs = W.b200_requests(w, device=dev)
        keep = m.select_many(reqs).cpu()
        agg = m.last_stats[3].cpu()
        for _ in range(3):  # several steps: the exchange's epochs advance
            assert torch.equal(m.select_many(reqs).cpu(), keep)
        m.compress_many(reqs)
        m.check_device_errors()
        torch.cuda.synchronize()
        dst = [torch.tensor(w.dst_tables[i]) for i in w.compressed()]
        pages = {f"{i}/{li}": (k[t.to(dev)].cpu(), v[t.to(dev)].cpu())
                 for li, (k, v) in enumerate(caches) for i, t in zip(w.compressed(), dst)}
        torch.save({"keep": keep, "pages": pages, "agg": agg, "mode": m.tp_sync_mode}, Path(out) / f"rank{rank}.pt")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_tp2_matches_tp1(mode, tmp_path):
    import torch.multiprocessing as mp

    import kvc_workloads as W

    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), mode), nprocs=2, start_method="spawn",
                       join=True)
    r0, r1 = (torch.load(tmp_path / f"rank{r}.pt") for r in (0, 1))
    assert r0["mode"] == r1["mode"] == mode
    assert torch.equal(r0["keep"], r1["keep"])
    assert torch.equal(r0["agg"].view(torch.int32), r1["agg"].view(torch.int32))
    w = _workload()
    caches = [tuple(t.cuda() for t in W.kv_pages(w, layer)) for layer in range(w.geometry.num_layers)]
    with tempfile.TemporaryDirectory() as d:
        m = W.b200_method(w, caches, W.write_stats_file(w, d))
    reqs = W.b200_requests(w)
    keep = m.select_many(reqs).cpu()
    assert torch.equal(keep, r0["keep"]), "TP=2 selection must equal TP=1 (MAX commutes with head sharding)"
    assert torch.equal(m.last_stats[3].cpu().view(torch.int32), r0["agg"].view(torch.int32))
    m.compress_many(reqs)
    torch.cuda.synchronize()
    per = w.geometry.num_kv_heads // 2
    for i in w.compressed():
        t = torch.tensor(w.dst_tables[i]).cuda()
        for li, (k, v) in enumerate(caches):
            for r, res in enumerate((r0, r1)):
                pk, pv = res["pages"][f"{i}/{li}"]
                assert torch.equal(k[t][:, :, r * per:(r + 1) * per].cpu().view(torch.int16), pk.view(torch.int16))
                assert torch.equal(v[t][:, :, r * per:(r + 1) * per].cpu().view(torch.int16), pv.view(torch.int16))

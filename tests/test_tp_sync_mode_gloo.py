"""Choice of the TP score-sync path, agreed by all ranks (gloo on CPU).

The peer-memory exchange is used only when every rank can reach every other
rank's memory; one rank without peer access (or a request for NCCL) sends the
whole group to the all-reduce path, so ranks never disagree on the protocol.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, str(ROOT / "vllm-ascend-kvcompress-hust_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from vllm_ascend_kvcompress.methods.triattention.tp_exchange import choose_tp_sync_mode

        g = dist.group.WORLD
        got = [choose_tp_sync_mode(g, rank, requested="peer", local_ok=True),
               choose_tp_sync_mode(g, rank, requested="peer", local_ok=rank == 0),
               choose_tp_sync_mode(g, rank, requested="nccl", local_ok=True),
               choose_tp_sync_mode(g, rank, requested="peer" if rank else "nccl", local_ok=True)]
        Path(out_dir, f"rank{rank}.txt").write_text(",".join(got))
    finally:
        dist.destroy_process_group()


def test_all_ranks_agree_on_the_sync_path(tmp_path):
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    for r in (0, 1):
        assert (tmp_path / f"rank{r}.txt").read_text() == "peer,nccl,nccl,nccl"


def test_exchange_layout_is_aligned_and_ordered():
    sys.path.insert(0, str(ROOT / "vllm-ascend-kvcompress-hust_b200"))
    from vllm_ascend_kvcompress.methods.triattention.tp_exchange import exchange_layout

    flags, agg, inbox, total = exchange_layout(8, 6, 1000, 26)
    # 250 quads over 8 ranks -> 32 per rank; inbox 8 sources x 6 layers x 32 quads x 16 B
    assert flags == 0 and agg == 256 and inbox == 256 + 4096 and total == inbox + 8 * 6 * 32 * 16
    assert all(x % 256 == 0 for x in (agg, inbox, total))


def test_exchange_buffers_grow_collectively_only_when_needed(monkeypatch):
    """ensure() rebuilds (a collective) only for a new layer count or more tokens than it holds."""
    sys.path.insert(0, str(ROOT / "vllm-ascend-kvcompress-hust_b200"))
    import torch

    from vllm_ascend_kvcompress.methods.triattention import tp_exchange as T

    calls = []

    def fake_rebuild(self, layers, cap):
        calls.append((layers, cap))
        self.layers, self.cap_tokens = layers, cap

    monkeypatch.setattr(T.PeerScoreExchange, "_rebuild", fake_rebuild)
    monkeypatch.setattr(T.N, "lib", lambda: type("L", (), {"kvc_tp_exchange_flag_words": staticmethod(lambda w: 2 * w + 1)})())
    ex = T.PeerScoreExchange(None, 0, 2, torch.device("cpu"))
    ex.ensure(6, 1000)
    ex.ensure(6, 900)       # fits
    ex.ensure(6, 1000)      # fits exactly
    ex.ensure(6, 1001)      # grows by at least 1.5x
    ex.ensure(5, 10)        # a new layer count always rebuilds
    assert calls == [(6, 1000), (6, 1500), (5, 128)]

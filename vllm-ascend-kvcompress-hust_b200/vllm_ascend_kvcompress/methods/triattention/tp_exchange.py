"""Tensor-parallel score sync over NVLink peer memory (CUDA IPC + two kernels).

The reference synchronises the per-layer head-max rows of a TP group with one
MAX all-reduce and then reduces the layers on every rank
(src/vllm_ascend_kvcompress/methods/triattention/method.py:447-467).  Here the
step's tokens are split into one range per rank; each rank's normalisation
stores its rows of every range straight into the owning rank's inbox (mapped
through CUDA IPC), and ``kvc_tp_exchange_max`` has each rank reduce its range
over all ranks' rows from its own inbox, reduce the layers, and store the
finished scores into every rank's agg buffer.  The scores are bit-identical to
the all-reduce path (MAX commutes with the head sharding; the layer reduction
is the same sequential code).

``PeerScoreExchange`` owns the buffers of one rank.  Growing them is a
collective: every rank of the group must call ``ensure`` with the same
arguments in the same step (they do, since the step's requests are the same
on every rank).
"""

from __future__ import annotations

import ctypes
import os

import torch

from ... import _native as N

_MODE_ENV = "KVC_B200_TP_SYNC"
_ALIGN = 256


def exchange_layout(world: int, layers: int, cap_tokens: int, flag_words: int) -> tuple[int, int, int, int]:
    """(flags, agg, inbox) byte offsets and total bytes of one rank's exchange buffer.

    The inbox holds [world source ranks][layers][quads per rank][4] fp32, for
    steps of up to ``cap_tokens`` page-padded tokens (quads of 4 tokens, split
    evenly over the ranks, as kvc_tp_exchange_inbox_floats sizes it).
    """
    up = lambda n: -(-n // _ALIGN) * _ALIGN
    flags = 0
    agg = up(flag_words * 4)
    inbox = agg + up(cap_tokens * 4)
    per = -(-(-(-cap_tokens // 4)) // world)
    return flags, agg, inbox, inbox + up(world * layers * per * 16)


def ipc_capable_allocator() -> bool:
    """CUDA IPC handles need cudaMalloc-backed memory (not expandable segments)."""
    conf = os.environ.get("PYTORCH_CUDA_ALLOC_CONF", "") + "," + os.environ.get("PYTORCH_ALLOC_CONF", "")
    return "expandable_segments:true" not in conf.replace(" ", "").lower()


def choose_tp_sync_mode(group, device_index: int, requested: str | None = None, local_ok=None) -> str:
    """"peer" when every rank can reach every other rank's memory, else "nccl".

    A collective over ``group``: every rank must call it, and all get the same answer.
    ``requested`` (default: the KVC_B200_TP_SYNC environment variable, else
    "peer") may force "nccl"; "peer" is only a request.  ``local_ok`` overrides
    this rank's own peer-access check (for tests without GPUs).
    """
    import torch.distributed as dist

    mode = (requested or os.environ.get(_MODE_ENV, "peer")).lower()
    if mode not in ("peer", "nccl"):
        raise ValueError(f"{_MODE_ENV} must be peer or nccl")
    world = dist.get_world_size(group)
    devices = [None] * world
    dist.all_gather_object(devices, int(device_index), group=group)
    if local_ok is None:
        lib = N.lib()
        local_ok = ipc_capable_allocator() and all(lib.kvc_can_access_peer(device_index, d) for d in devices)
    votes = [None] * world
    dist.all_gather_object(votes, bool(local_ok and mode == "peer" and world <= N.TP_MAX_WORLD), group=group)
    return "peer" if all(votes) else "nccl"


class PeerScoreExchange:
    """One rank's exchange buffers and the device tables of every rank's addresses."""

    def __init__(self, group, rank: int, world: int, device: torch.device) -> None:
        self.group = group
        self.rank = rank
        self.world = world
        self.device = device
        self.flag_words = int(N.lib().kvc_tp_exchange_flag_words(world))
        self.layers = 0
        self.cap_tokens = 0
        self.buf: torch.Tensor | None = None
        self.opened: list[int] = []
        self.table: torch.Tensor | None = None
        self.inbox_ptr = self.agg_ptr = 0
        self.epoch = 0

    def ensure(self, layers: int, tok_total: int) -> None:
        """Make room for ``layers`` rows of ``tok_total`` tokens (collective when it grows)."""
        if layers == self.layers and tok_total <= self.cap_tokens:
            return
        cap = max(tok_total, int(self.cap_tokens * 1.5) if layers == self.layers else 0, 128)
        self._rebuild(layers, cap)

    def _rebuild(self, layers: int, cap: int) -> None:
        import torch.distributed as dist

        lib = N.lib()
        dev = self.device.index
        # nobody may still read or write the old buffers; unmap the others'
        # before anyone lets go of its own
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.close()
        dist.barrier(group=self.group)
        self.buf = None
        flags_off, agg_off, inbox_off, total = exchange_layout(self.world, layers, cap, self.flag_words)
        buf = torch.zeros(total, dtype=torch.uint8, device=self.device)
        handle = (ctypes.c_char * N.IPC_HANDLE_BYTES)()
        off = ctypes.c_int64()
        N.check(lib.kvc_ipc_export(dev, buf.data_ptr(), handle, ctypes.byref(off)), "kvc_ipc_export")
        torch.cuda.synchronize(self.device)  # zeroed flags before any peer maps them
        got = [None] * self.world
        dist.all_gather_object(got, (bytes(handle), off.value), group=self.group)
        bases = []
        for p, (h, o) in enumerate(got):
            if p == self.rank:
                bases.append(buf.data_ptr())
                continue
            base = ctypes.c_void_p()
            hb = (ctypes.c_char * N.IPC_HANDLE_BYTES).from_buffer_copy(h)
            N.check(lib.kvc_ipc_open(dev, hb, ctypes.byref(base)), "kvc_ipc_open")
            self.opened.append(base.value)
            bases.append(base.value + o)
        self.table = torch.tensor([b + inbox_off for b in bases] + [b + agg_off for b in bases]
                                  + [b + flags_off for b in bases], dtype=torch.int64, device=self.device)
        self.buf = buf
        self.layers = layers
        self.cap_tokens = cap
        self.inbox_ptr = buf.data_ptr() + inbox_off
        self.agg_ptr = buf.data_ptr() + agg_off
        self._agg_off = agg_off
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def agg_view(self, tok_total: int) -> torch.Tensor:
        return self.buf[self._agg_off: self._agg_off + 4 * tok_total].view(torch.float32)

    def stamps_view(self) -> torch.Tensor:
        """This rank's four %globaltimer stamps of the last exchange (int64 ns, device):
        first CTA start, every rank ready, last CTA done, every rank's scores pushed."""
        w = int(N.lib().kvc_tp_exchange_stamp_word(self.world))
        return self.buf[4 * w: 4 * w + 32].view(torch.int64)

    def tables(self) -> tuple[int, int, int]:
        """Device addresses of the inbox, agg and flags tables (``world`` addresses each)."""
        t = self.table.data_ptr()
        return t, t + 8 * self.world, t + 16 * self.world

    def next_epoch(self) -> int:
        """The epoch of the next exchange (every rank advances it once per step)."""
        self.epoch += 1
        return self.epoch

    def close(self) -> None:
        """Unmap the other ranks' buffers (callers synchronise first); this rank's buffer stays."""
        lib = N.lib()
        for base in self.opened:
            lib.kvc_ipc_close(self.device.index, base)
        self.opened = []
        self.table = None

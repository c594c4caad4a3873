"""The peer-memory TP exchange kernels through the C ABI on one GPU.

world = 1 runs the whole data path against this rank's own buffers: rows
placed in the inbox (including NaN / +-inf values) and reduced by
kvc_tp_exchange_max must equal kvc_aggregate_rows bit for bit, and
kvc_tp_push_rows followed by the exchange must equal kvc_normalize_aggregate's
scores bit for bit; the exchange leaves its %globaltimer stamps in order.  A
world-2 call whose other rank never arrives must give up after its bounded
waits, report KVC_DEV_TIMEOUT and leave the context usable.  The two-GPU
exchange is covered by test_gpu_tp_nccl.py.
"""

from __future__ import annotations

import time

import pytest
import torch

from vllm_ascend_kvcompress import _native as N

pytestmark = pytest.mark.gpu


def _meta(lengths):
    pages = [-(-t // 128) for t in lengths]
    off = [0]
    for p in pages:
        off.append(off[-1] + p)
    tokens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    page_off = torch.tensor(off, dtype=torch.int32, device="cuda")
    return tokens, page_off, off[-1]


def _buffers(world, layers, pages):
    lib = N.lib()
    words = lib.kvc_tp_exchange_flag_words(world)
    inbox_n = lib.kvc_tp_exchange_inbox_floats(world, layers, pages)
    inbox = [torch.zeros(inbox_n, device="cuda") for _ in range(world)]
    agg = [torch.full((pages * 128,), 7.0, device="cuda") for _ in range(world)]
    flags = [torch.zeros(words, dtype=torch.int32, device="cuda") for _ in range(world)]
    table = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")
    return inbox, agg, flags, table(inbox), table(agg), table(flags)


@pytest.mark.parametrize("layer_agg", [N.AGG_MEAN, N.AGG_MAX])
def test_single_rank_exchange_equals_aggregate_rows_bitwise(layer_agg):
    lib = N.lib()
    lengths = [300, 1, 128, 2049]
    tokens, page_off, pages = _meta(lengths)
    tok, L = pages * 128, 5
    inbox, agg, flags, t_inbox, t_agg, t_flags = _buffers(1, L, pages)
    assert inbox[0].numel() == L * tok  # one rank owns every quad: the inbox is [L][tokens]
    g = torch.Generator(device="cuda").manual_seed(5)
    rows = torch.randn(L * tok, generator=g, device="cuda") * 3
    rows[17] = float("nan")
    rows[tok + 40] = float("inf")
    rows[2 * tok + 41] = float("-inf")
    inbox[0].copy_(rows)
    ref = torch.full((tok,), 3.0, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.kvc_aggregate_rows(rows.data_ptr(), L, pages, tokens.data_ptr(), page_off.data_ptr(),
                                  len(lengths), layer_agg, ref.data_ptr(), stream) == 0
    for epoch in (1, 2):  # two steps in a row: epochs advance, flags are never cleared
        agg[0].fill_(7.0)
        flags[0][0] = epoch  # this rank's rows are in its inbox ("delivered")
        assert lib.kvc_tp_exchange_max(t_inbox.data_ptr(), t_agg.data_ptr(), t_flags.data_ptr(), 1, 0, L, pages,
                                       tokens.data_ptr(), page_off.data_ptr(), len(lengths), layer_agg, epoch,
                                       err.data_ptr(), stream) == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(agg[0].view(torch.int32), ref.view(torch.int32))
    # delivered, pushed, exchange CTA counter, started epoch, push CTA counter
    assert flags[0].tolist()[:5] == [2, 2, 0, 2, 0]
    w0 = lib.kvc_tp_exchange_stamp_word(1)
    stamps = flags[0][w0: w0 + 8].view(torch.int64).tolist()
    assert 0 < stamps[0] <= stamps[1] <= stamps[2] <= stamps[3]


@pytest.mark.parametrize("heads,layer_agg", [(5, N.AGG_MEAN), (40, N.AGG_MAX)])
def test_single_rank_push_then_exchange_equals_normalize_aggregate(heads, layer_agg):
    lib = N.lib()
    lengths = [700, 2049, 5, 4096]
    tokens, page_off, pages = _meta(lengths)
    L, R = 3, len(lengths)
    g = torch.Generator(device="cuda").manual_seed(11 + heads)
    raw = torch.randn(L, pages, heads, 128, generator=g, device="cuda") * 4 + 1
    raw[1, 2, 0, 3] = float("nan")
    mean = torch.randn(L, R, heads, generator=g, device="cuda")
    den = torch.rand(L, R, heads, generator=g, device="cuda") * 2 + 1e-3
    stream = torch.cuda.current_stream().cuda_stream
    rows = torch.empty(L * pages * 128, device="cuda")
    ref = torch.empty(pages * 128, device="cuda")
    assert lib.kvc_normalize_aggregate(raw.data_ptr(), L, heads, pages, mean.data_ptr(), den.data_ptr(),
                                       tokens.data_ptr(), page_off.data_ptr(), R, layer_agg, rows.data_ptr(),
                                       ref.data_ptr(), stream) == 0
    inbox, agg, flags, t_inbox, t_agg, t_flags = _buffers(1, L, pages)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for epoch in (1, 2, 3):
        agg[0].fill_(7.0)
        assert lib.kvc_tp_push_rows(raw.data_ptr(), L, heads, pages, mean.data_ptr(), den.data_ptr(),
                                    tokens.data_ptr(), page_off.data_ptr(), R, t_inbox.data_ptr(), t_flags.data_ptr(),
                                    1, 0, epoch, stream) == 0
        assert lib.kvc_tp_exchange_max(t_inbox.data_ptr(), t_agg.data_ptr(), t_flags.data_ptr(), 1, 0, L, pages,
                                       tokens.data_ptr(), page_off.data_ptr(), R, layer_agg, epoch, err.data_ptr(),
                                       stream) == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(agg[0].view(torch.int32), ref.view(torch.int32))
    assert flags[0].tolist()[:2] == [3, 3]


def test_exchange_rejects_bad_arguments_on_the_host():
    lib = N.lib()
    tokens, page_off, pages = _meta([256])
    _, _, _, t_inbox, t_agg, t_flags = _buffers(1, 1, pages)
    s = torch.cuda.current_stream().cuda_stream
    args = lambda world, rank, epoch: (t_inbox.data_ptr(), t_agg.data_ptr(), t_flags.data_ptr(), world, rank, 1,
                                       pages, tokens.data_ptr(), page_off.data_ptr(), 1, N.AGG_MEAN, epoch, None, s)
    assert lib.kvc_tp_exchange_max(*args(1, 1, 1)) == -22  # rank outside the world
    assert lib.kvc_tp_exchange_max(*args(0, 0, 1)) == -22
    assert lib.kvc_tp_exchange_max(*args(1, 0, 0)) == -22  # epochs start at 1
    f = torch.zeros(1, device="cuda")
    assert lib.kvc_tp_push_rows(f.data_ptr(), 1, 1, pages, f.data_ptr(), f.data_ptr(), tokens.data_ptr(),
                                page_off.data_ptr(), 1, t_inbox.data_ptr(), t_flags.data_ptr(), 1, 1, 1, s) == -22


def test_absent_rank_times_out_with_an_error_status():
    """Rank 1 never arrives: both bounded waits expire, the flag reports it, the GPU stays usable."""
    lib = N.lib()
    tokens, page_off, pages = _meta([1000])
    inbox, agg, flags, t_inbox, t_agg, t_flags = _buffers(2, 2, pages)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    flags[0][0] = 1  # this rank's own rows delivered; rank 1's never are
    t0 = time.perf_counter()
    assert lib.kvc_tp_exchange_max(t_inbox.data_ptr(), t_agg.data_ptr(), t_flags.data_ptr(), 2, 0, 2, pages,
                                   tokens.data_ptr(), page_off.data_ptr(), 1, N.AGG_MEAN, 1, err.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(err.item()) & N.DEV_TIMEOUT
    assert 1.5 < waited < 30
    # this rank gave up, still signalled "pushed" to the absent one, and gave up waiting for its signal
    assert flags[1].tolist()[2] == 1 and flags[1].tolist()[0] == 0
    x = torch.arange(10, device="cuda")
    assert int(x.sum()) == 45

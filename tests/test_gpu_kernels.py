"""GPU known-answer and golden tests of the individual kernels through the C ABI.

Known answers restate the literal cases of the reference's tests
(tests/test_scoring.py, test_selection.py, test_cache.py, run_npu_kernel_smoke.py);
golden selections come from running the reference's select_keep_indices.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import kvc_workloads as W
from cases import golden
from oracle import triattention_oracle as O
from vllm_ascend_kvcompress import _native as N
from vllm_ascend_kvcompress.calibration import LayerAccumulator
from vllm_ascend_kvcompress.methods.triattention import kernels as K
from vllm_ascend_kvcompress.methods.triattention.cache import (
    gather_paged_tokens,
    materialize_selected_tokens,
    materialize_token_slots,
    token_slots,
)
from vllm_ascend_kvcompress.methods.triattention.selection import select_keep_indices

pytestmark = pytest.mark.gpu
dev = "cuda"


# ---- selection -----------------------------------------------------------


def test_selection_matches_reference_golden():
    arrays, spec = golden()
    cases = spec["selection"]
    scores = W.golden_selection_scores(cases)
    for n, (t, b, p, r, s, pol) in enumerate(cases):
        keep = select_keep_indices(scores[n].to(dev), budget=b, protected_prefix=p, protected_recent=r,
                                   segments=s, policy=pol)
        assert np.array_equal(keep.cpu().numpy(), arrays[f"selection/{n}/keep"]), (t, b, p, r, s, pol)


def test_selection_known_answers():
    keep = select_keep_indices(torch.arange(16, dtype=torch.float32, device=dev), budget=12, protected_prefix=2,
                               protected_recent=2, segments=4, policy="v3")
    assert set(range(16)) - set(keep.tolist()) == {2, 5, 8, 11}
    keep = select_keep_indices(torch.tensor([10.0, 9.0, 8.0, 7.0, -5.0, -6.0], device=dev), budget=4,
                               protected_prefix=0, protected_recent=2, segments=8, policy="global")
    assert keep.tolist() == [0, 1, 4, 5]
    keep = select_keep_indices(torch.zeros(19, device=dev), budget=13, protected_prefix=2, protected_recent=2,
                               segments=8, policy="v3")
    assert keep.numel() == 13 and {0, 1, 17, 18} <= set(keep.tolist())


def test_selection_ties_take_lowest_positions():
    scores = torch.zeros(1000, device=dev)
    keep = select_keep_indices(scores, budget=300, protected_prefix=0, protected_recent=0, segments=1,
                               policy="v3").tolist()
    assert keep == list(range(300))
    s = torch.tensor([1.0, 5.0, 5.0, 5.0, 0.0, 5.0, 2.0], device=dev)
    keep = select_keep_indices(s, budget=3, protected_prefix=0, protected_recent=0, segments=1, policy="global")
    assert keep.tolist() == [1, 2, 3]


def test_selection_special_values_and_validation():
    s = torch.tensor([float("-inf"), 1e30, -1.0, 3.0, float("-inf"), 0.5, -0.0, 0.0], device=dev)
    keep = select_keep_indices(s, budget=4, protected_prefix=0, protected_recent=0, segments=1, policy="v3")
    assert keep.tolist() == [1, 3, 5, 7] or keep.tolist() == [1, 3, 5, 6]
    with pytest.raises(ValueError, match="budget"):
        select_keep_indices(s, budget=9, protected_prefix=0, protected_recent=0, segments=1, policy="v3")
    with pytest.raises(ValueError, match="protected"):
        select_keep_indices(s, budget=4, protected_prefix=3, protected_recent=2, segments=1, policy="v3")


@pytest.mark.parametrize("t,b,p,r,s", [(65536, 4608, 128, 512, 8), (50000, 49999, 0, 0, 7), (4736, 4608, 128, 512, 8),
                                       (9000, 1000, 0, 0, 1), (3000, 2000, 1000, 1000, 8)])
def test_selection_random_vs_oracle(t, b, p, r, s):
    g = torch.Generator().manual_seed(t + b)
    scores = torch.randn(t, generator=g)
    ref = O.select_keep_indices(scores, budget=b, protected_prefix=p, protected_recent=r, segments=s, policy="v3")
    got = select_keep_indices(scores.to(dev), budget=b, protected_prefix=p, protected_recent=r, segments=s,
                              policy="v3")
    assert torch.equal(got.cpu(), ref)


# ---- paged cache API -----------------------------------------------------


def test_gather_maps_logical_tokens_through_block_table():
    cache = torch.arange(12, dtype=torch.float32, device=dev).view(3, 4, 1, 1)
    got = gather_paged_tokens(cache, torch.tensor([2, 0], device=dev), torch.tensor([0, 3, 4, 7], device=dev), 4)
    assert got.flatten().tolist() == [8.0, 11.0, 0.0, 3.0]


def test_materialize_overlapping_destination_gathers_first():
    k = torch.arange(16, dtype=torch.float32, device=dev).view(4, 4, 1, 1)
    v = k.clone() + 100
    src, keep = torch.tensor([2, 0, 3], device=dev), torch.tensor([1, 4, 6, 9], device=dev)
    ek = gather_paged_tokens(k, src, keep, 4).clone()
    ev = gather_paged_tokens(v, src, keep, 4).clone()
    materialize_selected_tokens(k, v, src, torch.tensor([2], device=dev), keep, 4)
    torch.testing.assert_close(k[2], ek)
    torch.testing.assert_close(v[2], ev)


def test_padded_interleaved_pages_keep_unused_bytes():
    bs, nb, heads, dim = 4, 4, 1, 2
    page = bs * heads * dim
    stride = 2 * page + 4
    raw = torch.full((nb * stride,), -1, dtype=torch.float16, device=dev)
    shape, strides = (nb, bs, heads, dim), (stride, heads * dim, dim, 1)
    k = torch.as_strided(raw, shape, strides)
    v = torch.as_strided(raw, shape, strides, storage_offset=page)
    k.copy_(torch.arange(nb * page, device=dev).view(shape))
    v.copy_(torch.arange(nb * page, device=dev).view(shape) + 100)
    src, keep = torch.tensor([2, 0, 3], device=dev), torch.tensor([1, 4, 6, 9], device=dev)
    ek = gather_paged_tokens(k, src, keep, bs).clone()
    ev = gather_paged_tokens(v, src, keep, bs).clone()
    materialize_selected_tokens(k, v, src, torch.tensor([2], device=dev), keep, bs)
    torch.testing.assert_close(k[2], ek)
    torch.testing.assert_close(v[2], ev)
    s_slots = token_slots(torch.tensor([2], device=dev), torch.arange(4, device=dev), bs)
    d_slots = token_slots(torch.tensor([1], device=dev), torch.arange(4, device=dev), bs)
    materialize_token_slots(k, v, s_slots, d_slots, torch.empty_like(ek), torch.empty_like(ev))
    torch.testing.assert_close(k[1], ek)
    torch.testing.assert_close(v[1], ev)
    torch.testing.assert_close(raw.view(nb, stride)[:, -4:], torch.full((nb, 4), -1, dtype=torch.float16, device=dev))


def test_gather_slot_out_of_range_is_flagged():
    cache = torch.zeros(3, 4, 1, 2, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    K.gather_slots(cache, torch.tensor([0, 12, 5], device=dev), error_flag=flag)
    assert int(flag) & N.DEV_BLOCK_RANGE


def test_shift_positions_known_answer():
    out = torch.empty(3, dtype=torch.int64, device=dev)
    K.shift_positions(torch.tensor([300, 20, 301], device=dev), torch.tensor([0, 1, 0], device=dev),
                      torch.tensor([172, 0], device=dev), out)
    assert out.tolist() == [128, 20, 129]
    K.shift_positions(torch.tensor([300, 20, 301], device=dev), torch.tensor([0, 1, 0], device=dev, dtype=torch.int32),
                      torch.tensor([172, 0], device=dev), out)
    assert out.tolist() == [128, 20, 129]


# ---- scoring known answers (embedded in an 8-frequency paged cache) ------


def _score_small(keys: torch.Tensor, qr, qi, qabs, fsq, omega, rot_small: int, q_pass=None, round_start: int = 1,
                 offsets=(1.0,)):
    """Score tiny half-RoPE keys ``[T, 1, D]`` by zero-padding F to 8 and P to 8 (zeros add nothing)."""
    T, _, d = keys.shape
    f_small = rot_small // 2
    p_small = d - rot_small
    F, P = 8, (8 if p_small else 0)
    D = 2 * F + P
    G = qr.shape[1]
    padded = torch.zeros(T, 1, D)
    padded[:, 0, :f_small] = keys[:, 0, :f_small]
    padded[:, 0, F:F + f_small] = keys[:, 0, f_small:rot_small]
    if p_small:
        padded[:, 0, 2 * F:2 * F + p_small] = keys[:, 0, rot_small:]
    pages = -(-T // 128)
    cache = torch.zeros(pages, 128, 1, D, dtype=torch.bfloat16)
    cache.view(-1, 1, D)[:T] = padded.to(torch.bfloat16)
    cache = cache.to(dev)

    def pad_f(t):
        out = torch.zeros(1, G, F)
        out[..., :f_small] = t
        return out

    omega_p = torch.zeros(F)
    omega_p[:f_small] = omega
    scale = torch.sqrt(pad_f(fsq))
    qmag = torch.sqrt(pad_f(qr).square() + pad_f(qi).square() + 1e-8)
    extra = pad_f(qabs) - qmag
    extra[..., f_small:] = 0.0
    meta = torch.tensor([T, 0, pages], dtype=torch.int32, device=dev)
    i64 = torch.tensor([0, pages, 0, 1, round_start, round_start], dtype=torch.int64, device=dev)
    plan = K.BatchPlan(1, pages, meta[:1], meta[1:], torch.arange(pages, device=dev), i64[:2], i64[:0], i64[2:4],
                       i64[4:5], i64[5:6], (T,), 0)
    offs = torch.tensor(offsets, device=dev)
    coef = torch.empty(K.coef_floats(F, G, offs.numel(), N.AGG_MEAN), device=dev)
    K.prepare_score_coefficients(omega_p[None].to(dev).contiguous(), offs, plan, pad_f(qr)[None].to(dev).contiguous(),
                                 pad_f(qi)[None].to(dev).contiguous(), scale[None].to(dev).contiguous(),
                                 extra[None].to(dev).contiguous(), N.AGG_MEAN, coef)
    qp = None
    if p_small:
        qpp = torch.zeros(1, G, P)
        qpp[..., :p_small] = q_pass
        qp = qpp.transpose(-1, -2).contiguous()[None].to(dev).contiguous()
    raw = torch.empty(G * pages * 128, device=dev)
    part = torch.empty(pages * G * 2, device=dev)
    K.score_paged_keys(N.pointer_array([cache.data_ptr()]), torch.bfloat16, cache.stride(0), pages, 1, G, D,
                       2 * F, plan, coef, offs.numel(), N.AGG_MEAN, qp, raw, part, None)
    return raw.view(G, -1)[:, :T].cpu()


def test_score_query_side_scale_gives_four():
    got = _score_small(torch.tensor([[[2.0, 0.0]]]), torch.ones(1, 1, 1), torch.zeros(1, 1, 1), torch.ones(1, 1, 1),
                       torch.full((1, 1, 1), 4.0), torch.zeros(1), rot_small=2)
    torch.testing.assert_close(got, torch.tensor([[4.0]]))


def test_score_partial_rope_content_term():
    got = _score_small(torch.tensor([[[0.0, 0.0, 3.0, 4.0]], [[0.0, 0.0, -2.0, 1.0]]]), torch.zeros(1, 1, 1),
                       torch.zeros(1, 1, 1), torch.zeros(1, 1, 1), torch.ones(1, 1, 1), torch.zeros(1), rot_small=2,
                       q_pass=torch.tensor([[[2.0, -1.0]]]))
    torch.testing.assert_close(got, torch.tensor([[2.0, -5.0]]))


def test_score_mean_over_offsets_matches_oracle():
    keys = torch.tensor([[[1.0, 2.0, 3.0, 4.0]], [[0.5, 1.5, 2.5, 3.5]], [[2.0, 1.0, 4.0, 3.0]]])
    st = O.LayerStats(torch.tensor([[[1.0, 0.5], [0.25, 0.75]]]), torch.tensor([[[0.0, 0.5], [0.5, 0.25]]]),
                      torch.ones(1, 2, 2), torch.ones(1, 2, 2), torch.tensor([1.0, 0.1]))
    ref = O.score_keys(keys, st, round_start=3, offsets=torch.tensor([1.0, 2.0, 4.0]))[0]
    got = _score_small(keys, st.q_mean_real, st.q_mean_imag, st.q_abs_mean, st.freq_scale_sq, st.omega, rot_small=4,
                       round_start=3, offsets=(1.0, 2.0, 4.0))
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)


# ---- calibration ------------------------------------------------------------


@pytest.mark.parametrize("case", ["calib_full", "calib_partial"])
def test_calibration_matches_reference_golden(case):
    arrays, spec = golden()
    inputs = {n: (h, d, r, q) for n, h, d, r, q in W.golden_calibration_inputs()}
    heads, hd, rot, calls = inputs[case]
    acc = LayerAccumulator()
    for q in calls:
        acc.add(q.to(dev), heads, hd, rot)
    assert acc.count == spec[case]["count"]
    for k in ("real_sum", "imag_sum", "abs_sum", "pass_sum"):
        key = f"{case}/{k}"
        if key in arrays:
            torch.testing.assert_close(getattr(acc, k).float().cpu(), torch.from_numpy(arrays[key]), rtol=1e-5, atol=1e-4)


def test_calibration_large_vs_fp64_and_packed_gate():
    heads, hd, rot = 40, 128, 128
    q = W.calibration_queries(0, 2, 8192, heads, hd, device=dev)
    acc = LayerAccumulator()
    acc.add(q[:10000], heads, hd, rot)
    gate = torch.cat([q[10000:], torch.randn_like(q[10000:])], dim=1)  # Qwen3.5 packs the gate after Q
    acc.add(gate, heads, hd, rot)
    v = q.cpu().double().reshape(-1, heads, hd)
    re, im = v[..., : rot // 2], v[..., rot // 2: rot]
    want_all = {"q_mean_real": re.mean(0), "q_mean_imag": im.mean(0),
                "q_abs_mean": torch.sqrt(re.square() + im.square()).mean(0)}
    mean_abs = v.abs().mean().item()
    got = acc.means()
    for k, want in want_all.items():
        err = (got[k].double() - want).abs().max().item()
        assert err <= 1e-4 * max(want.abs().max().item(), mean_abs), (k, err)


def test_calibration_partial_rope_unaligned_widths():
    heads, hd, rot = 3, 20, 6  # F = 3, P = 14: falls back to narrow vectors
    q = torch.randn(777, heads * hd, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    acc = LayerAccumulator()
    acc.add(q.to(dev), heads, hd, rot)
    ref = O.CalibrationSums()
    ref.add(q.double(), heads, hd, rot)
    torch.testing.assert_close(acc.real_sum.float().cpu(), ref.real_sum, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(acc.abs_sum.float().cpu(), ref.abs_sum, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(acc.pass_sum.float().cpu(), ref.pass_sum, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("heads,layer_agg", [(5, N.AGG_MEAN), (40, N.AGG_MEAN), (40, N.AGG_MAX), (1, N.AGG_MAX)])
def test_normalize_aggregate_equals_torch_bitwise_with_near_ties(heads, layer_agg):
    """Normalise + head max + layer reduction: rows and agg equal torch fp32 bit for bit, also where
    several heads' quotients are within an ulp of each other."""
    lib = N.lib()
    lengths = [300, 2049, 128, 5000, 1]
    pages = [-(-t // 128) for t in lengths]
    off = [0]
    for p in pages:
        off.append(off[-1] + p)
    P, L, R = off[-1], 4, len(lengths)
    g = torch.Generator(device="cuda").manual_seed(40 + heads)
    raw = torch.randn(L, P, heads, 128, generator=g, device="cuda") * 5 + 2
    mean = torch.randn(L, R, heads, generator=g, device="cuda")
    den = torch.rand(L, R, heads, generator=g, device="cuda") * 3 + 1e-3
    req = torch.repeat_interleave(torch.arange(R, device="cuda"), torch.tensor(pages, device="cuda"))
    if heads > 1:  # near ties: every head's quotient within a few ulps of head 0's on a band of tokens
        mu, dn = mean[:, req, :, None], den[:, req, :, None]
        q0 = (raw[:, :, :1] - mu[:, :, :1]) / dn[:, :, :1]
        nudge = torch.randint(-3, 4, raw.shape, generator=g, device="cuda").float() * 2.0 ** -22
        tied = q0 * (1 + nudge) * dn + mu
        band = torch.zeros(128, dtype=torch.bool, device="cuda")
        band[::3] = True
        raw = torch.where(band, tied, raw)
        raw[0, 0, :, 0] = raw[0, 0, 0, 0]  # exact duplicates
    raw[0, 3, 0, 7] = float("nan")
    raw[1, 2, heads - 1, 9] = float("inf")
    raw[2, 5, 0, 0] = float("-inf")
    tokens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    page_off = torch.tensor(off, dtype=torch.int32, device="cuda")
    mu, dn = mean[:, req, :, None], den[:, req, :, None]
    ref_rows = ((raw - mu) / dn).amax(dim=2).reshape(L, P * 128)
    pos = torch.arange(P * 128, device="cuda")
    start = torch.repeat_interleave(torch.tensor(off[:-1], device="cuda"), torch.tensor(pages, device="cuda")) * 128
    valid = (pos - start.repeat_interleave(128)) < tokens[req].long().repeat_interleave(128)
    ref_rows = torch.where(valid[None], ref_rows, torch.zeros_like(ref_rows))
    acc = ref_rows[0].clone()
    for layer in range(1, L):
        acc = acc + ref_rows[layer] if layer_agg == N.AGG_MEAN else torch.maximum(acc, ref_rows[layer])
    if layer_agg == N.AGG_MEAN:
        acc = acc / L
    ref_agg = torch.where(valid, acc.nan_to_num(nan=float("-inf"), posinf=1e30, neginf=float("-inf")),
                          torch.zeros_like(acc))
    stream = torch.cuda.current_stream().cuda_stream
    rows = torch.full((L, P * 128), 123.0, device="cuda")
    agg = torch.full((P * 128,), 7.0, device="cuda")
    assert lib.kvc_normalize_aggregate(raw.data_ptr(), L, heads, P, mean.data_ptr(), den.data_ptr(),
                                       tokens.data_ptr(), page_off.data_ptr(), R, layer_agg, rows.data_ptr(),
                                       agg.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(agg.view(torch.int32), ref_agg.view(torch.int32))
    nan = torch.isnan(ref_rows)
    assert torch.equal(torch.isnan(rows), nan)
    assert torch.equal(rows[~nan].view(torch.int32), ref_rows[~nan].view(torch.int32))


@pytest.mark.parametrize("heads", [1, 3, 5, 40])
def test_normalize_rows_equal_torch_fp32_bitwise(heads):
    """kvc_normalize_aggregate rows == max over heads of (raw - mean) / den in IEEE fp32 (torch), padding 0."""
    lib = N.lib()
    lengths = [1, 300, 2049, 128, 5000]
    pages = [-(-t // 128) for t in lengths]
    off = [0]
    for p in pages:
        off.append(off[-1] + p)
    P, L, R = off[-1], 3, len(lengths)
    g = torch.Generator(device="cuda").manual_seed(heads)
    raw = torch.randn(L, P, heads, 128, generator=g, device="cuda") * 5 + 2
    raw[0, 3, 0, 7] = float("nan")
    raw[1, 2, heads - 1, 9] = float("inf")
    raw[2, 5, 0, 0] = float("-inf")
    mean = torch.randn(L, R, heads, generator=g, device="cuda")
    den = torch.rand(L, R, heads, generator=g, device="cuda") * 3 + 1e-3
    tokens = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    page_off = torch.tensor(off, dtype=torch.int32, device="cuda")
    rows = torch.full((L, P * 128), 123.0, device="cuda")
    assert lib.kvc_normalize_aggregate(raw.data_ptr(), L, heads, P, mean.data_ptr(), den.data_ptr(),
                                       tokens.data_ptr(), page_off.data_ptr(), R, N.AGG_MEAN, rows.data_ptr(),
                                       None, torch.cuda.current_stream().cuda_stream) == 0
    req = torch.repeat_interleave(torch.arange(R, device="cuda"), torch.tensor(pages, device="cuda"))  # per page
    mu = mean[:, req, :, None]  # [L, P, heads, 1]
    dn = den[:, req, :, None]
    ref = ((raw - mu) / dn).amax(dim=2).reshape(L, P * 128)
    pos = torch.arange(128, device="cuda").repeat(P) + 0
    valid = pos + (torch.arange(P, device="cuda") - page_off[req].long()).repeat_interleave(128) * 128 \
        < tokens[req].long().repeat_interleave(128)
    ref = torch.where(valid[None], ref, torch.zeros_like(ref))
    torch.cuda.synchronize()
    nan = torch.isnan(ref)
    assert nan.any() and torch.equal(torch.isnan(rows), nan)
    assert torch.equal(rows[~nan].view(torch.int32), ref[~nan].view(torch.int32))


@pytest.mark.parametrize("heads,parts", [(1, 4), (5, 4), (40, 4), (40, 1), (200, 4), (40, 8), (5, 8)])
def test_head_stats_match_fp64_var_mean(heads, parts):
    """kvc_head_stats from per-partial (sum, M2) equals torch.var_mean(correction=0) in fp64 within 1e-5."""
    lib = N.lib()
    lengths = [1, 129, 2049, 5000]
    pages = [-(-t // 128) for t in lengths]
    off = [0]
    for p in pages:
        off.append(off[-1] + p)
    P, L, R, span = off[-1], 2, len(lengths), 128 // parts
    g = torch.Generator().manual_seed(heads + parts)
    raw = torch.randn(L, heads, P * 128, generator=g, dtype=torch.float64) * 3 + 50  # large mean, small spread
    part = torch.zeros(L, P * parts, heads, 2, dtype=torch.float64)
    ref_mean = torch.empty(L, R, heads, dtype=torch.float64)
    ref_var = torch.empty(L, R, heads, dtype=torch.float64)
    for r, t in enumerate(lengths):
        x = raw[:, :, off[r] * 128: off[r] * 128 + t]
        ref_var[:, r], ref_mean[:, r] = torch.var_mean(x, dim=-1, correction=0)
        for q in range(-(-t // span)):
            seg = x[:, :, q * span: min(t, (q + 1) * span)]
            part[:, off[r] * parts + q, :, 0] = seg.sum(-1)
            part[:, off[r] * parts + q, :, 1] = ((seg - seg.mean(-1, keepdim=True)) ** 2).sum(-1)
    dev = lambda a, dt: a.to(dtype=dt).contiguous().cuda()
    partial = dev(part, torch.float32)
    out = [torch.empty(L * R * heads, device="cuda") for _ in range(3)]
    assert lib.kvc_head_stats(partial.data_ptr(), L, R, P, parts, heads,
                              dev(torch.tensor(lengths), torch.int32).data_ptr(),
                              dev(torch.tensor(off), torch.int32).data_ptr(), *(o.data_ptr() for o in out),
                              torch.cuda.current_stream().cuda_stream) == 0
    mean, var, den = (o.cpu().double().view(L, R, heads) for o in out)
    torch.testing.assert_close(mean, ref_mean, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(var, ref_var, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(den, ref_var.clamp_min(1e-6).sqrt(), rtol=1e-5, atol=1e-6)


def test_compaction_over_more_layers_than_one_launch_holds():
    """kvc_compact splits more than 512 layers into several launches with the same result."""
    blocks, rb = 12, 128 * 2 * 64 * 2  # 2 KV heads x head_dim 64 x bf16
    g = torch.Generator(device="cuda").manual_seed(9)
    k = torch.randn(blocks, 128, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(blocks, 128, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    T, budget = 700, 256
    src = torch.tensor([3, 7, 1, 9, 0, 5], dtype=torch.int64, device="cuda")
    dst = torch.tensor([10, 11], dtype=torch.int64, device="cuda")
    keep = torch.sort(torch.randperm(T, generator=torch.Generator().manual_seed(2))[:budget]).values.cuda()
    meta = torch.tensor([T, 0, -(-T // 128)], dtype=torch.int32, device="cuda")
    i64 = torch.tensor([0, src.numel(), 0, dst.numel(), T, T], dtype=torch.int64, device="cuda")
    plan = K.BatchPlan(1, -(-T // 128), meta[:1], meta[1:], src, i64[:2], dst, i64[2:4], i64[4:5], i64[5:6],
                       (T,), dst.numel())
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    expect_k, expect_v = k.clone(), v.clone()
    slots = (src[keep // 128] * 128 + keep % 128)
    out = (dst[torch.arange(budget, device="cuda") // 128] * 128 + torch.arange(budget, device="cuda") % 128)
    expect_k.view(-1, 2, 64)[out] = k.view(-1, 2, 64)[slots]
    expect_v.view(-1, 2, 64)[out] = v.view(-1, 2, 64)[slots]
    n = 520  # the same cache pair named 520 times: every layer writes the same rows
    K.compact(N.pointer_array([k.data_ptr()] * n), N.pointer_array([v.data_ptr()] * n), k.stride(0) * 2, blocks,
              rb // 128, plan, keep, budget, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(k.view(torch.int16), expect_k.view(torch.int16))
    assert torch.equal(v.view(torch.int16), expect_v.view(torch.int16))


@pytest.mark.parametrize("kvh,head_dim", [(4, 128), (8, 256), (24, 256), (1, 8)])
def test_compaction_row_widths(kvh, head_dim):
    """1 KB, 4 KB and 12 KB rows (bulk copies; 12 KB is the largest they take) and 16-byte rows."""
    blocks = 10
    g = torch.Generator(device="cuda").manual_seed(kvh * head_dim)
    k = torch.randn(blocks, 128, kvh, head_dim, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(blocks, 128, kvh, head_dim, generator=g, device="cuda").to(torch.bfloat16)
    T, budget = 600, 200
    src = torch.tensor([4, 0, 7, 2, 9], dtype=torch.int64, device="cuda")
    dst = torch.tensor([8, 6], dtype=torch.int64, device="cuda")
    keep = torch.sort(torch.randperm(T, generator=torch.Generator().manual_seed(kvh))[:budget]).values.cuda()
    meta = torch.tensor([T, 0, -(-T // 128)], dtype=torch.int32, device="cuda")
    i64 = torch.tensor([0, src.numel(), 0, dst.numel(), T, T], dtype=torch.int64, device="cuda")
    plan = K.BatchPlan(1, -(-T // 128), meta[:1], meta[1:], src, i64[:2], dst, i64[2:4], i64[4:5], i64[5:6],
                       (T,), dst.numel())
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    expect_k, expect_v = k.clone(), v.clone()
    slots = src[keep // 128] * 128 + keep % 128
    j = torch.arange(budget, device="cuda")
    out = dst[j // 128] * 128 + j % 128
    expect_k.view(-1, kvh, head_dim)[out] = k.view(-1, kvh, head_dim)[slots]
    expect_v.view(-1, kvh, head_dim)[out] = v.view(-1, kvh, head_dim)[slots]
    row_bytes = kvh * head_dim * 2
    K.compact(N.pointer_array([k.data_ptr()] * 3), N.pointer_array([v.data_ptr()] * 3), k.stride(0) * 2, blocks,
              row_bytes, plan, keep, budget, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(k.view(torch.int16), expect_k.view(torch.int16))
    assert torch.equal(v.view(torch.int16), expect_v.view(torch.int16))

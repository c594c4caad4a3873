"""CPU oracle for the TriAttention score -> select -> compact path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this file.
It is used by ``tests/`` as the parity checker, by ``__graft_entry__.smoke()``
as the checker of one small GPU invocation, and by ``bench.py``'s CPU-baseline
leg (``--impl reference`` and the ``cpu_baseline`` object).  It must never be
the thing that is measured as the GPU product or shipped as a fallback.

It restates, in PyTorch CPU fp32 operations, the algorithm of the reference
plugin ``vllm-ascend-kvcompress-hust`` 0.10.0 (paths below are relative to that
project's root).  The reference is itself a torch program; on a non-NPU device
it runs exactly this CPU op sequence, so the restatement keeps the op order
wherever rounding matters (phase formation, cos/sin means, products, sums,
var_mean, normalisation, layer accumulation).  Parity of this file with the
reference is pinned by ``tests/golden/make_golden.py`` (which imports the real
reference) and ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch

BLOCK = 128


# ---------------------------------------------------------------------------
# scoring  (src/vllm_ascend_kvcompress/methods/triattention/scoring.py)
# ---------------------------------------------------------------------------


def geometric_offsets(maximum: int) -> torch.Tensor:
    """Future-query offsets 1, 2, 4, ... <= maximum (scoring.py:11-20)."""
    if maximum < 1:
        raise ValueError("maximum scoring offset must be positive")
    values = []
    v = 1
    while v <= maximum:
        values.append(float(v))
        v *= 2
    return torch.tensor(values, dtype=torch.float32)


@dataclass(frozen=True)
class LayerStats:
    """Per-layer calibration grouped by KV head: tensors are [kvh, G, F] fp32.

    Mirrors DeviceLayerCalibrationStats (stats.py:42-51).
    """

    q_mean_real: torch.Tensor
    q_mean_imag: torch.Tensor
    q_abs_mean: torch.Tensor
    freq_scale_sq: torch.Tensor
    omega: torch.Tensor  # [F]
    rotary_dim: int | None = None
    q_pass_mean: torch.Tensor | None = None  # [kvh, G, P]
    rope_style: str = "half"

    def shard(self, rank: int, size: int) -> "LayerStats":
        """KV-head shard of one TP rank (stats.py:315-323)."""
        kvh = self.q_mean_real.shape[0]
        if kvh % size:
            raise ValueError("kv heads must divide by TP size")
        lo = rank * (kvh // size)
        hi = lo + kvh // size
        return LayerStats(
            self.q_mean_real[lo:hi].contiguous(),
            self.q_mean_imag[lo:hi].contiguous(),
            self.q_abs_mean[lo:hi].contiguous(),
            self.freq_scale_sq[lo:hi].contiguous(),
            self.omega,
            self.rotary_dim,
            None if self.q_pass_mean is None else self.q_pass_mean[lo:hi].contiguous(),
            self.rope_style,
        )


def score_keys(
    keys: torch.Tensor,
    stats: LayerStats,
    *,
    round_start: int,
    offsets: torch.Tensor,
    aggregation: str = "mean",
) -> torch.Tensor:
    """Trigonometric score of post-RoPE keys ``[T, kvh, D]`` -> ``[kvh, G, T]``.

    Follows score_post_rope_keys (scoring.py:23-120): per frequency f the key
    is split "half" style into (k[f], k[F+f]); the calibrated mean query is
    rotated by the mean over future offsets of cos/sin((off + rs) * omega_f);
    the |k| * (E|q| - |E q|) term and, for partial RoPE, the direct q_pass . k
    content term are added.
    """
    t, kvh, d = keys.shape
    rot = d if stats.rotary_dim is None else stats.rotary_dim
    f = rot // 2
    kf = keys.to(torch.float32).permute(1, 0, 2)
    rk = kf[..., :rot]
    if stats.rope_style == "interleaved":
        kr, ki = rk[..., 0::2], rk[..., 1::2]
    else:
        kr, ki = rk[..., :f], rk[..., f:rot]
    qr = stats.q_mean_real.unsqueeze(2)
    qi = stats.q_mean_imag.unsqueeze(2)
    kr = kr.unsqueeze(1)
    ki = ki.unsqueeze(1)
    pr = qr * kr + qi * ki
    pi = qi * kr - qr * ki
    scale = torch.sqrt(stats.freq_scale_sq).unsqueeze(2)
    # scoring.py:77 -- fp32 (offset + round_start) then * omega
    phases = (offsets.unsqueeze(1) + float(round_start)) * stats.omega.unsqueeze(0)
    if aggregation == "mean":
        c = torch.cos(phases).mean(dim=0).view(1, 1, 1, f)
        s = torch.sin(phases).mean(dim=0).view(1, 1, 1, f)
        out = (scale * (pr * c - pi * s)).sum(dim=-1)
    elif aggregation == "max":
        out = torch.full((kvh, qr.shape[1], t), float("-inf"), dtype=torch.float32)
        for ph in phases.unbind(0):
            c = torch.cos(ph).view(1, 1, 1, f)
            s = torch.sin(ph).view(1, 1, 1, f)
            out = torch.maximum(out, (scale * (pr * c - pi * s)).sum(dim=-1))
    else:
        raise ValueError(f"unsupported score aggregation: {aggregation}")
    kabs = torch.sqrt(kr.square() + ki.square())
    qabs = torch.sqrt(stats.q_mean_real.square() + stats.q_mean_imag.square() + 1e-8)
    extra = (stats.q_abs_mean - qabs).unsqueeze(2)
    out = out + (kabs * extra * scale).sum(dim=-1)
    if rot < d:
        if stats.q_pass_mean is None:
            raise ValueError("partial-RoPE scoring requires q_pass_mean")
        kp = kf[..., rot:].unsqueeze(1)
        out = out + (stats.q_pass_mean.unsqueeze(2) * kp).sum(dim=-1)
    return out


def normalize_head_scores(raw: torch.Tensor, mean: torch.Tensor, var: torch.Tensor) -> torch.Tensor:
    """z-score per query head along tokens (scoring.py:123-128)."""
    return (raw - mean.unsqueeze(-1)) / torch.sqrt(var.clamp_min(1e-6)).unsqueeze(-1)


# ---------------------------------------------------------------------------
# selection  (src/vllm_ascend_kvcompress/methods/triattention/selection.py)
# ---------------------------------------------------------------------------


def v3_segments(token_count: int, budget: int, prefix: int, recent: int, segments: int):
    """Integer V3 plan: list of (start, stop, keep_count) (selection.py:160-190).

    Segment s covers [P0 + M*s//S, P0 + M*(s+1)//S); its eviction quota is the
    difference of E*(offset)//M at both ends, so quotas sum exactly to E.
    """
    p0 = prefix
    m = token_count - prefix - recent
    e = token_count - budget
    if e > m:
        raise ValueError("selection budget leaves too few slots for protected tokens")
    plan = []
    for s in range(segments):
        start = p0 + m * s // segments
        stop = p0 + m * (s + 1) // segments
        n = stop - start
        if n == 0:
            plan.append((start, stop, 0))
            continue
        ev = e * (stop - p0) // m - e * (start - p0) // m
        plan.append((start, stop, n - ev))
    return plan


def select_keep_indices(
    scores: torch.Tensor,
    *,
    budget: int,
    protected_prefix: int,
    protected_recent: int,
    segments: int,
    policy: str,
) -> torch.Tensor:
    """Sorted int64 keep positions (selection.py:108-196, CPU branch)."""
    if scores.ndim != 1:
        raise ValueError("scores must be one-dimensional")
    t = int(scores.numel())
    if budget <= 0 or budget > t:
        raise ValueError("budget must be in [1, token_count]")
    if protected_prefix < 0 or protected_recent < 0:
        raise ValueError("protected windows must be non-negative")
    if protected_prefix + protected_recent > budget:
        raise ValueError("protected windows cannot exceed the selection budget")
    if segments <= 0:
        raise ValueError("segments must be positive")
    prefix = min(protected_prefix, t)
    recent = min(protected_recent, t - prefix)
    protected = torch.zeros(t, dtype=torch.bool)
    protected[:prefix] = True
    if recent:
        protected[t - recent:] = True
    if policy == "global":
        ranked = scores.clone()
        ranked[protected] = float("inf")
        top = torch.topk(ranked, k=budget, largest=True, sorted=False).indices
        return torch.sort(top).values
    if policy != "v3":
        raise ValueError(f"unsupported position policy: {policy}")
    keep = protected.clone()
    for start, stop, k in v3_segments(t, budget, prefix, recent, segments):
        n = stop - start
        if n == 0 or k <= 0:
            continue
        if k == n:
            keep[start:stop] = True
            continue
        local = torch.topk(scores[start:stop], k=k, largest=True, sorted=False).indices
        keep[start + local] = True
    out = torch.nonzero(keep, as_tuple=False).flatten()
    if out.numel() != budget:
        raise RuntimeError(f"V3 selected {out.numel()} tokens, expected exactly {budget}")
    return out


def selection_boundaries(
    scores: torch.Tensor, keep: torch.Tensor, *, budget: int, prefix: int, recent: int,
    segments: int, policy: str,
) -> list[tuple[int, int, float]]:
    """(start, stop, threshold) per selected range: the lowest kept score.

    Used by parity tests to decide whether a differing index is a near-tie.
    """
    t = scores.numel()
    prefix = min(prefix, t)
    recent = min(recent, t - prefix)
    mask = torch.zeros(t, dtype=torch.bool)
    mask[keep] = True
    if policy == "global":
        ranges = [(prefix, t - recent)]
    else:
        ranges = [(a, b) for a, b, k in v3_segments(t, budget, prefix, recent, segments) if 0 < k < b - a]
    out = []
    for a, b in ranges:
        seg = scores[a:b]
        kept = seg[mask[a:b]]
        if kept.numel() and kept.numel() < seg.numel():
            out.append((a, b, float(kept.min())))
    return out


# ---------------------------------------------------------------------------
# paged cache  (src/vllm_ascend_kvcompress/methods/triattention/cache.py)
# ---------------------------------------------------------------------------


def token_slots(block_ids: torch.Tensor, idx: torch.Tensor, block: int = BLOCK) -> torch.Tensor:
    """Logical token -> flat physical slot (cache.py:9-15)."""
    return block_ids.index_select(0, torch.div(idx, block, rounding_mode="floor")) * block + idx % block


def gather_slots(cache: torch.Tensor, slots: torch.Tensor) -> torch.Tensor:
    """Rows ``cache[slot // bs, slot % bs]`` for any page stride (cache.py:18-33)."""
    bs = cache.shape[1]
    return cache[torch.div(slots, bs, rounding_mode="floor"), slots % bs]


def write_slots(cache: torch.Tensor, slots: torch.Tensor, values: torch.Tensor) -> None:
    """Scatter rows into slots (cache.py:36-45)."""
    bs = cache.shape[1]
    cache[torch.div(slots, bs, rounding_mode="floor"), slots % bs] = values


def gather_paged_range(cache, block_ids, start: int, count: int, block: int = BLOCK):
    """Contiguous logical range through the block table (cache.py:61-76)."""
    return gather_slots(cache, token_slots(block_ids, torch.arange(start, start + count), block))


def materialize(k_cache, v_cache, src_blocks, dst_blocks, keep, block: int = BLOCK) -> None:
    """Gather kept rows, then write them densely into destination blocks.

    cache.py:79-111 (gather fully before writing, so overlapping source and
    destination blocks are safe).
    """
    src = token_slots(src_blocks, keep, block)
    dst = token_slots(dst_blocks, torch.arange(keep.numel()), block)
    gk = gather_slots(k_cache, src).clone()
    gv = gather_slots(v_cache, src).clone()
    write_slots(k_cache, dst, gk)
    write_slots(v_cache, dst, gv)


# ---------------------------------------------------------------------------
# method orchestration  (method.py:256-503)
# ---------------------------------------------------------------------------


@dataclass
class OracleRequest:
    semantic_num_tokens: int
    physical_num_tokens: int
    src_blocks: torch.Tensor  # int64 kernel block ids
    dst_blocks: torch.Tensor


@dataclass
class OracleOptions:
    kv_budget: int
    protected_prefix_window: int = 0
    protected_recent_window: int = 128
    position_segments: int = 8
    position_policy: str = "v3"
    score_aggregation: str = "mean"
    layer_aggregation: str = "mean"
    score_chunk_size: int = 8192
    score_layer_stride: int = 8


def layer_rows(
    k_caches: Sequence[torch.Tensor],
    stats: Sequence[LayerStats],
    req: OracleRequest,
    opts: OracleOptions,
    offsets: torch.Tensor,
    *,
    keep_raw: bool = False,
):
    """Per scoring layer, max over local heads of the normalised scores.

    method.py:340-446: layers sampled with ``score_layer_stride``; each scored
    in ``score_chunk_size`` chunks (gather + score_post_rope_keys); torch
    var_mean (population); normalise; amax over (kv head, q head).
    Returns ``[L_s, T]`` fp32 (and raw/mean/var per layer when asked).
    """
    t = req.physical_num_tokens
    rows = []
    extras = []
    for kc, st in list(zip(k_caches, stats))[:: opts.score_layer_stride]:
        pieces = []
        for a in range(0, t, opts.score_chunk_size):
            n = min(opts.score_chunk_size, t - a)
            keys = gather_paged_range(kc, req.src_blocks, a, n)
            pieces.append(
                score_keys(keys, st, round_start=req.semantic_num_tokens,
                           offsets=offsets, aggregation=opts.score_aggregation)
            )
        raw = torch.cat(pieces, dim=-1)
        var, mean = torch.var_mean(raw, dim=-1, correction=0)
        rows.append(normalize_head_scores(raw, mean, var).amax(dim=(0, 1)))
        if keep_raw:
            extras.append((raw, mean, var))
    out = torch.stack(rows)
    return (out, extras) if keep_raw else out


def aggregate_rows(rows: torch.Tensor, layer_aggregation: str) -> torch.Tensor:
    """Layer reduction + finalise (method.py:458-467): sum or max, mean, nan_to_num."""
    n = rows.shape[0]
    if layer_aggregation == "mean":
        agg = rows[0].clone()
        for i in range(1, n):
            agg.add_(rows[i])
        agg.div_(float(n))
    else:
        agg = rows[0].clone()
        for i in range(1, n):
            torch.maximum(agg, rows[i], out=agg)
    return agg.nan_to_num_(nan=float("-inf"), posinf=1e30, neginf=float("-inf"))


def select_request(k_caches, stats, req: OracleRequest, opts: OracleOptions, offsets,
                   tp_size: int = 1):
    """Scores -> keep indices for one request (method.py:297-475).

    With ``tp_size > 1`` the KV heads are split into ``tp_size`` shards, each
    shard produces its own per-layer rows and the rows are combined by an
    elementwise MAX -- the all-reduce of method.py:453-457.
    """
    if tp_size == 1:
        rows = layer_rows(k_caches, stats, req, opts, offsets)
    else:
        kvh = k_caches[0].shape[2]
        per = kvh // tp_size
        shards = []
        for r in range(tp_size):
            kc = [c[:, :, r * per:(r + 1) * per] for c in k_caches]
            st = [s.shard(r, tp_size) for s in stats]
            shards.append(layer_rows(kc, st, req, opts, offsets))
        rows = shards[0]
        for s in shards[1:]:
            rows = torch.maximum(rows, s)
    agg = aggregate_rows(rows, opts.layer_aggregation)
    keep = select_keep_indices(
        agg, budget=opts.kv_budget, protected_prefix=opts.protected_prefix_window,
        protected_recent=opts.protected_recent_window, segments=opts.position_segments,
        policy=opts.position_policy,
    )
    return agg, keep


def compress_request(k_caches, v_caches, stats, req: OracleRequest, opts: OracleOptions,
                     offsets, tp_size: int = 1):
    """Full pass for one request: select, then compact every layer (method.py:256-295)."""
    agg, keep = select_request(k_caches, stats, req, opts, offsets, tp_size)
    for kc, vc in zip(k_caches, v_caches):
        materialize(kc, vc, req.src_blocks, req.dst_blocks, keep)
    return agg, keep


# ---------------------------------------------------------------------------
# calibration reduction  (src/vllm_ascend_kvcompress/calibration.py:87-131)
# ---------------------------------------------------------------------------


@dataclass
class CalibrationSums:
    real_sum: torch.Tensor | None = None
    imag_sum: torch.Tensor | None = None
    abs_sum: torch.Tensor | None = None
    pass_sum: torch.Tensor | None = None
    count: int = 0

    def add(self, q: torch.Tensor, heads: int, head_dim: int, rotary_dim: int) -> None:
        """Accumulate one batch of pre-RoPE queries ``[..., heads*head_dim]``.

        calibration.py:95-131: per (head, frequency) sums of the real part
        q[:F], imaginary part q[F:rot], modulus sqrt(re^2 + im^2), and per
        (head, pass dim) sums of q[rot:], all in fp32; count = rows seen.
        """
        v = q.detach().reshape(-1, heads, head_dim).float()
        f = rotary_dim // 2
        re, im, ps = v[..., :f], v[..., f:rotary_dim], v[..., rotary_dim:]
        rs, is_, ab = re.sum(0), im.sum(0), torch.sqrt(re.square() + im.square()).sum(0)
        self.real_sum = rs if self.real_sum is None else self.real_sum + rs
        self.imag_sum = is_ if self.imag_sum is None else self.imag_sum + is_
        self.abs_sum = ab if self.abs_sum is None else self.abs_sum + ab
        if ps.numel():
            p = ps.sum(0)
            self.pass_sum = p if self.pass_sum is None else self.pass_sum + p
        self.count += v.shape[0]

    def means(self):
        """Mean stats as written into the schema-3 payload (calibration.py:349-360)."""
        d = float(self.count)
        out = {
            "q_mean_real": self.real_sum / d,
            "q_mean_imag": self.imag_sum / d,
            "q_abs_mean": self.abs_sum / d,
        }
        if self.pass_sum is not None:
            out["q_pass_mean"] = self.pass_sum / d
        return out


def shift_positions(positions, request_indices, request_offsets):
    """Physical decode positions (kernels.py:35-47): pos - offsets[req]."""
    return positions - request_offsets.index_select(0, request_indices.to(torch.long))


def stats_from_payload(payload: dict, num_kv_heads: int, group: int, rotary_dim: int,
                       layers: Sequence[int]) -> list[LayerStats]:
    """LayerStats per layer from a schema-3 payload whose rows are per query head.

    Query heads are grouped kv-major ``[kvh, G, F]`` as stats.py:345-360 does.
    """
    out = []
    g = lambda t: t.float().reshape(num_kv_heads, group, -1).contiguous()
    for li in layers:
        e = payload["layer_stats"][str(li)]
        out.append(LayerStats(
            q_mean_real=g(e["q_mean_real"]), q_mean_imag=g(e["q_mean_imag"]), q_abs_mean=g(e["q_abs_mean"]),
            freq_scale_sq=g(e["freq_scale_sq"]), omega=e["inv_freq"].float().contiguous(), rotary_dim=rotary_dim,
            q_pass_mean=g(e["q_pass_mean"]) if "q_pass_mean" in e else None))
    return out

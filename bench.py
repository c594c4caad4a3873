"""Benchmark of the B200 TriAttention score -> select -> compact pass.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--stride 8|1]
                    [--config 0|1|2|3|4] [--no-other-configs] [--no-cpu-baseline]

Headline workload (N = 1): the Qwen2.5-14B-shaped ragged batch of the
benchmark specification (config 1): 48 layers, 40 query / 8 KV heads, head_dim
128, RoPE theta 1e6, BF16 K/V ~ N(0, 1), 128-token pages placed by a seeded
permutation, 32 sequences of U[4096, 32768] tokens (seed 1), kv_budget 4608,
recompute window 128, V3 policy (prefix 128, recent 512, 8 segments), mean/mean
aggregation, score_layer_stride 8.  One step = one score + select + compact
pass over every compressed sequence and every layer.  Inputs (~145 GB of K/V)
are far larger than L2, so no flush is needed between steps.

N > 1 (torchrun, one process per GPU): the same batch with the 8 KV heads
sharded over N tensor-parallel ranks; every step runs one score sync over the
ranks (strong scaling: total work fixed).

Every run checks its own results outside the timed region: the median-length
request's scores, keep indices and compacted K/V bytes (first and last layer)
against the CPU oracle fed with the run's own K/V, and at N > 1 that every rank
holds identical keep indices ("parity" in the JSON line).  The default run also
measures the specification's other configurations ("other_configs"): configs
0, 2, 3 and 4 at N = 1, config 2 (TP = 2 as specified) and config 4 at N = 2,
config 4 at N = 4 and 8.

--impl reference times the CPU oracle (a restatement of the reference's own
torch CPU path) on a bounded sample of the same workload, with all host cores.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass, replace
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "vllm-ascend-kvcompress-hust_b200"))

import torch  # noqa: E402

import kvc_workloads as W  # noqa: E402

METRIC = "KV tokens scored+compacted/s per GPU & % HBM roofline; TP score-sync µs at 2/4/8"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0
SCORE_TOL = 1e-3  # |d| <= 1e-3 * max(|ref|, 1) on fp32 scores
L2_BYTES = 126 * 2 ** 20


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(w: W.Workload, kv_heads: int) -> dict[str, float]:
    """Bytes the pass must move (excludes implementation round trips such as raw scores).

    scoring: every scoring layer reads each compressed token's K once
             (L_s * T * kvh * D * 2); the score row of each layer is written
             once (L_s * T * 4).
    compaction: every layer reads and writes the kept K and V rows
             (N * B * kvh * D * 2 * 2 (K, V) * 2 (read + write)).
    selection: the final score row is read and B int64 indices written.
    """
    g = w.geometry
    o = w.options
    ls = -(-g.num_layers // o.score_layer_stride)
    T = w.total_compressed_tokens()
    R = len(w.compressed())
    row = kv_heads * g.head_dim * 2
    return {
        "score": ls * T * row + ls * T * 4.0,
        "compact": g.num_layers * R * o.kv_budget * row * 2 * 2.0,
        "select": T * 4.0 + R * o.kv_budget * 8.0,
    }


class StageTimer:
    """CUDA events recorded at each pipeline stage boundary on the current stream."""

    def __init__(self) -> None:
        self.steps: list[list[tuple[str, torch.cuda.Event]]] = []
        self.active = False
        self.stamps: list[torch.Tensor] = []  # per step: the exchange kernel's four %globaltimer stamps

    def exchange_done(self, ex) -> None:
        """Keep a device copy of the peer exchange's stamps of this step (read after the pass)."""
        if self.active:
            self.stamps.append(ex.stamps_view().clone())

    def exchange_us(self) -> dict | None:
        """Median rank-skew wait and exchange time inside the exchange kernel (this rank's clock)."""
        if not self.stamps:
            return None
        t = torch.stack(self.stamps).cpu().double()
        wait = (t[:, 1] - t[:, 0]) / 1e3
        exch = (t[:, 3] - t[:, 1]) / 1e3
        total = (t[:, 3] - t[:, 0]) / 1e3
        med = lambda x: float(x.median())
        return {"tp_wait_us": med(wait), "tp_exchange_us": med(exch), "tp_kernel_us": med(total),
                "steps": int(t.shape[0])}

    def new_step(self) -> None:
        if self.active:
            self.steps.append([])

    def mark(self, name: str) -> None:
        if not self.active:
            return
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.steps[-1].append((name, ev))

    def add(self, name: str, ev: torch.cuda.Event) -> None:
        """Take an event the library records at a stage boundary inside one native call."""
        if self.active:
            self.steps[-1].append((name, ev))

    def stage_ms(self) -> dict[str, float]:
        """Median duration of each stage (from its mark to the next mark) over the steps."""
        acc: dict[str, list[float]] = {}
        for marks in self.steps:
            for (name, a), (_, b) in zip(marks, marks[1:]):
                acc.setdefault(name, []).append(a.elapsed_time(b))
        return {k: sorted(v)[len(v) // 2] for k, v in acc.items()}


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(tempfile.mkstemp(suffix=".csv")[1])

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

WORKLOAD_TEXT = {
    "config0": "config0: CPU-runnable reference op, 1 layer, 40 q / 8 kv heads, head_dim 128, 4 seqs "
               "{{1000, 2500, 4096, 6000}}, kv_budget 2048, V3 prefix 4 / recent 128",
    "config1": "config1: Qwen2.5-14B-shaped ragged batch, {layers} layers, 40 q / 8 kv heads, head_dim 128, "
               "{seqs} seqs U[4096,32768] (seed 1), kv_budget 4608, V3 prefix 128 / recent 512 / 8 segments",
    "config2": "config2: Qwen3.5-35B-A3B-shaped full-attention layers, 10 layers, 16 q / 2 kv heads, head_dim 256, "
               "partial RoPE 64, 2048-token pages, 16 seqs U[8192,53248] (seed 2), kv_budget 4608, stride 2",
    "config4": "config4: 48 layers ({distinct} distinct caches aliased round-robin), 40 q / 8 kv heads, head_dim 128, "
               "{seqs} seqs U[2048,65536] (seed 4), kv_budget 4608, stride 8",
}


def make_workload(config: int, args) -> W.Workload:
    if config == 0:
        return W.config0()
    if config == 2:
        return W.config2()
    if config == 4:
        return W.config4(num_seqs=args.seqs if args.seqs != 32 else 128, stride=args.stride)
    return W.config1(stride=args.stride, num_seqs=args.seqs, num_layers=args.layers)


def distinct_layers(config: int, args, w: W.Workload) -> int:
    if args.distinct_layers:
        return min(args.distinct_layers, w.geometry.num_layers)
    return 5 if config == 4 else w.geometry.num_layers


def config_dict(w: W.Workload, world: int, distinct: int | None = None) -> dict:
    o = w.options
    kv_bytes = 2 * w.num_blocks * W.BLOCK * w.geometry.num_kv_heads * w.geometry.head_dim * 2 * (
        distinct or w.geometry.num_layers)
    return {
        "workload": WORKLOAD_TEXT[w.name].format(layers=w.geometry.num_layers, seqs=len(w.lengths),
                                                 distinct=distinct or w.geometry.num_layers),
        "global_batch": len(w.lengths), "compressed_sequences": len(w.compressed()),
        "compressed_tokens": w.total_compressed_tokens(), "layers": w.geometry.num_layers,
        "score_layer_stride": o.score_layer_stride, "kv_budget": o.kv_budget,
        "parallelism": f"tp{world}" if world > 1 else "single",
        "l2": ("inputs ({:.0f} GB of K/V) exceed L2; no flush needed".format(kv_bytes / 1e9) if kv_bytes > 4 * L2_BYTES
               else "L2 flushed (256 MB write) before every timed step; up to 3 (flush, step) pairs queued "
                    "behind a ~1 ms device spin so the device time excludes host launch time"),
    }


# ---------------------------------------------------------------------------
# oracle leg: the CPU baseline and the result check (the oracle is the checker)
# ---------------------------------------------------------------------------


def oracle_inputs(w: W.Workload):
    from oracle import triattention_oracle as O

    geo, o = w.geometry, w.options
    stats = O.stats_from_payload(W.calibration_payload(geo, w.seed), geo.num_kv_heads, geo.group, geo.rotary_dim,
                                 range(geo.num_layers))
    opts = O.OracleOptions(kv_budget=o.kv_budget, protected_prefix_window=o.protected_prefix_window,
                           protected_recent_window=o.protected_recent_window, position_segments=o.position_segments,
                           position_policy=o.position_policy, score_aggregation=o.score_aggregation,
                           layer_aggregation=o.layer_aggregation, score_chunk_size=o.score_chunk_size,
                           score_layer_stride=o.score_layer_stride)
    return stats, opts, O.geometric_offsets(o.max_model_len)


def near_tie_count(w: W.Workload, ref_agg, ref_keep, got_keep) -> tuple[int, int]:
    """(#differing indices, #of them whose oracle score is NOT within the tolerance of its segment's boundary)."""
    from oracle import triattention_oracle as O

    diff = sorted(set(ref_keep.tolist()) ^ set(got_keep.tolist()))
    if not diff:
        return 0, 0
    o = w.options
    bounds = O.selection_boundaries(ref_agg, ref_keep, budget=o.kv_budget, prefix=o.protected_prefix_window,
                                    recent=o.protected_recent_window, segments=o.position_segments,
                                    policy=o.position_policy)
    bad = 0
    for idx in diff:
        thr = [t for a, b, t in bounds if a <= idx < b]
        if not thr or abs(float(ref_agg[idx]) - thr[0]) > SCORE_TOL * max(abs(thr[0]), 1.0):
            bad += 1
    return len(diff), bad


def score_error(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max |got - ref| / (tol * max(|ref|, 1)) over finite entries; inf if the non-finite patterns differ."""
    finite = torch.isfinite(ref)
    if not torch.equal(finite, torch.isfinite(got)):
        return float("inf")
    if not bool(finite.any()):
        return 0.0
    err = (got[finite] - ref[finite]).abs() / (SCORE_TOL * ref[finite].abs().clamp_min(1.0))
    return float(err.max())


@dataclass
class Sample:
    """The median-length request's data from the run, on the host (all TP shards joined by head)."""
    index: int                 # sequence index in the workload
    tokens: int
    k_src: dict                # scoring/compaction layer -> [pages, 128, kvh, D]
    v_src: dict
    k_dst: dict                # compaction-checked layer -> GPU result [dst pages, 128, kvh, D]
    v_dst: dict
    keep: torch.Tensor         # GPU keep indices [B]
    agg: torch.Tensor          # GPU final scores [tokens]
    ranks_identical: bool | None


def collect_sample(ctx, w: W.Workload, m, physical, nd: int) -> Sample:
    """Gather the median request's K/V pages, GPU keep/scores and every rank's keep checksum (collective)."""
    comp = w.compressed()
    R = len(comp)
    j = sorted(range(R), key=lambda q: w.lengths[comp[q]])[R // 2]
    i = comp[j]
    T = w.lengths[i]
    n = -(-T // W.BLOCK)
    g, o = w.geometry, w.options
    scoring = list(range(0, g.num_layers, o.score_layer_stride))
    compact = sorted({0, g.num_layers - 1})
    src = torch.tensor(w.src_tables[i][:n], dtype=torch.long, device=ctx.dev)
    dst = torch.tensor(w.dst_tables[i], dtype=torch.long, device=ctx.dev)
    torch.cuda.synchronize()

    def joined(t: torch.Tensor) -> torch.Tensor:
        if ctx.world == 1:
            return t.cpu()
        import torch.distributed as dist

        parts = [torch.empty_like(t) for _ in range(ctx.world)]
        dist.all_gather(parts, t.contiguous())
        return torch.cat(parts, dim=2).cpu() if ctx.rank == 0 else torch.empty(0)

    k_src = {l: joined(physical[l % nd][0][src]) for l in sorted(set(scoring) | set(compact))}
    v_src = {l: joined(physical[l % nd][1][src]) for l in compact}
    k_dst = {l: joined(physical[l % nd][0][dst]) for l in compact}
    v_dst = {l: joined(physical[l % nd][1][dst]) for l in compact}
    keep_all = m._keep_view(R).view(R, o.kv_budget)
    keep = keep_all[j].cpu()
    off = sum(-(-w.lengths[q] // W.BLOCK) for q in comp[:j]) * W.BLOCK
    agg = m.last_stats[3][off: off + T].cpu()
    same = None
    if ctx.world > 1:
        import torch.distributed as dist

        # a position-weighted checksum of the whole step's keep workspace
        wts = torch.arange(1, keep_all.numel() + 1, device=ctx.dev, dtype=torch.int64).view_as(keep_all)
        ck = torch.stack([(keep_all * wts).sum(), keep_all.sum(), (keep_all * keep_all).sum()])
        got = [torch.empty_like(ck) for _ in range(ctx.world)]
        dist.all_gather(got, ck)
        same = all(torch.equal(x, got[0]) for x in got)
    return Sample(i, T, k_src, v_src, k_dst, v_dst, keep, agg, same)


def oracle_mini_caches(s: Sample, layer: int, dst_pages: int):
    """Host K/V caches of one layer: the request's source pages then blank destination pages."""
    blank = lambda t: torch.zeros((dst_pages,) + tuple(t.shape[1:]), dtype=t.dtype)
    return torch.cat([s.k_src[layer], blank(s.k_src[layer])]), torch.cat([s.v_src[layer], blank(s.v_src[layer])])


def parity_check(ctx, w: W.Workload, s: Sample) -> dict:
    """The oracle's scores, keep set and compaction for the sampled request vs the GPU's (rank 0)."""
    from oracle import triattention_oracle as O

    g, o = w.geometry, w.options
    torch.set_num_threads(os.cpu_count() or 1)  # torchrun defaults ranks to one thread
    stats, opts, offs = oracle_inputs(w)
    n = -(-s.tokens // W.BLOCK)
    dp = len(w.dst_tables[s.index])
    first = min(s.k_src)
    k_list = [s.k_src.get(l, s.k_src[first]) for l in range(g.num_layers)]  # unscored layers are never read
    req = O.OracleRequest(s.tokens, s.tokens, torch.arange(n), torch.arange(n, n + dp))
    ref_agg, ref_keep = O.select_request(k_list, stats, req, opts, offs, tp_size=ctx.world)
    diff, bad = near_tie_count(w, ref_agg, ref_keep, s.keep)
    rows = o.kv_budget
    bytes_equal = True
    for l in s.k_dst:
        kc, vc = oracle_mini_caches(s, l, dp)
        O.materialize(kc, vc, req.src_blocks, req.dst_blocks, s.keep)
        flat = lambda t: t.reshape(-1, *t.shape[2:])[:rows].view(torch.int16)
        bytes_equal &= torch.equal(flat(kc[n:]), flat(s.k_dst[l])) and torch.equal(flat(vc[n:]), flat(s.v_dst[l]))
    err = score_error(s.agg, ref_agg)
    sorted_ok = bool((s.keep[1:] > s.keep[:-1]).all())
    out = {
        "request": s.index, "tokens": s.tokens, "tp_size": ctx.world,
        "scores_max_err_over_tol": err, "scores_within_tol": err <= 1.0,
        "keep_match": bad == 0 and sorted_ok and s.keep.numel() == o.kv_budget, "keep_differing": diff,
        "near_ties": diff - bad, "bytes_equal": bool(bytes_equal), "layers_compaction_checked": sorted(s.k_dst),
        "ranks_identical": s.ranks_identical,
    }
    out["ok"] = bool(out["scores_within_tol"] and out["keep_match"] and out["bytes_equal"]
                     and s.ranks_identical is not False)
    return out


def cpu_baseline(w: W.Workload, s: Sample, repeats: int = 5) -> dict:
    """The oracle's full pass (score every scoring layer, select, compact all layers) on the sampled request."""
    from oracle import triattention_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = w.geometry
    stats, opts, offs = oracle_inputs(w)
    n = -(-s.tokens // W.BLOCK)
    dp = len(w.dst_tables[s.index])
    first = min(s.k_src)
    k_list = [s.k_src.get(l, s.k_src[first]) for l in range(g.num_layers)]
    copies = [oracle_mini_caches(s, l, dp) for l in sorted(s.v_src)]
    req = O.OracleRequest(s.tokens, s.tokens, torch.arange(n), torch.arange(n, n + dp))
    times = []
    for _ in range(repeats + 1):  # the first pass warms up
        t0 = time.perf_counter()
        _, keep = O.select_request(k_list, stats, req, opts, offs)
        for l in range(g.num_layers):
            kc, vc = copies[l % len(copies)]
            O.materialize(kc, vc, req.src_blocks, req.dst_blocks, keep)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times[1:])
    return {"value": s.tokens / t, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"oracle (torch CPU restatement of the reference path) on the median-length request "
                       f"({s.tokens} tokens) with this run's own K/V: {len(range(0, g.num_layers, opts.score_layer_stride))} "
                       f"scoring layers, selection, and compaction of all {g.num_layers} layers (aliased onto "
                       f"{len(copies)} host copies); median of {repeats} after a warm-up"),
            "seconds": t}


def run_cpu_sample(w: W.Workload, seq: int, distinct_layers: int = 8, repeats: int = 1) -> tuple[float, dict]:
    """The reference arm: the oracle on one sequence with all layers, from host-seeded K/V."""
    from oracle import triattention_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sw = W.place_blocks(W.Workload(w.name + "-cpu-sample", w.geometry, w.options, [w.lengths[seq]], seed=w.seed,
                                   cache_blocks_per_page=w.cache_blocks_per_page))
    geo = sw.geometry
    nd = min(distinct_layers, geo.num_layers)
    distinct = [W.kv_pages(sw, layer) for layer in range(nd)]
    caches = [distinct[i % nd] for i in range(geo.num_layers)]  # layer aliasing (same work)
    stats, opts, offs = oracle_inputs(sw)
    req = O.OracleRequest(sw.lengths[0], sw.lengths[0], torch.tensor(sw.src_tables[0]), torch.tensor(sw.dst_tables[0]))
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        _, keep = O.select_request([c[0] for c in caches], stats, req, opts, offs)
        for kc, vc in caches:
            O.materialize(kc, vc, req.src_blocks, req.dst_blocks, keep)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    desc = (f"oracle (torch CPU restatement of the reference path) on 1 sequence of {sw.lengths[0]} tokens, "
            f"all {geo.num_layers} layers (aliased onto {nd} distinct caches), "
            f"stride {opts.score_layer_stride}, median of {repeats}")
    return sw.lengths[0] / t, {"threads": threads, "seconds": t, "sample": desc}


def reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    w = make_workload(args.config, args)
    seq = sorted(w.compressed(), key=lambda i: w.lengths[i])[len(w.compressed()) // 2]  # median-length sequence
    budget_s = 150.0
    t0 = time.perf_counter()
    run_cpu_sample(w, seq)  # warm-up (one step)
    step_s = time.perf_counter() - t0
    steps = max(5, min(args.steps, int(budget_s / max(step_s, 1e-3))))
    value, info = run_cpu_sample(w, seq, repeats=steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": 1, "ms_per_step": info["seconds"] * 1e3, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) BF16 K/V, random calibration stats)",
        "config": config_dict(w, world, distinct_layers(args.config, args, w)),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": info["threads"], "kind": "port",
                         "sample": info["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------


@dataclass
class Ctx:
    rank: int
    world: int
    local: int
    dev: torch.device
    group: object


def barrier(ctx: Ctx) -> None:
    if ctx.world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(ctx: Ctx, x: float) -> float:
    if ctx.world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device=ctx.dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


# Small steps are shorter on the GPU than their launches take on the host, so
# timed back to back the GPU would mostly wait for the host.  Their device time
# is taken with up to QUEUED (flush, step) pairs queued behind a ~1 ms
# device-side spin, so the step's kernels run back to back as the events time
# them; the host's share stays in the end-to-end figure.
QUEUED = 3


def host_ahead() -> None:
    torch.cuda.synchronize()
    torch.cuda._sleep(2_000_000)  # clock cycles on the device: ~1 ms


class L2Flush:
    """Writes a 256 MB buffer (twice the L2) so the next step starts with a cold L2."""

    def __init__(self, dev) -> None:
        self.buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    def __call__(self) -> None:
        self.buf.fill_(1.0)


def release(ctx: Ctx, m) -> None:
    """Unmap the peer exchange buffers of a method before it is dropped (collective)."""
    torch.cuda.synchronize()
    barrier(ctx)
    if getattr(m, "_peer", None) is not None:
        m._peer.close()
    barrier(ctx)


def measure(ctx: Ctx, w: W.Workload, nd: int, steps: int, warmup: int, *, clocks: bool = False,
            check: bool = True, cpu: bool = True, flush: bool = False) -> dict:
    """Device-timed steps, a per-stage pass, the end-to-end pass, and the result check of one workload."""
    geo = w.geometry
    if geo.num_kv_heads % ctx.world:
        raise SystemExit(f"{geo.num_kv_heads} KV heads cannot be sharded over {ctx.world} ranks")
    kvh = geo.num_kv_heads // ctx.world
    physical = [W.kv_pages(w, layer * ctx.world + ctx.rank, kv_heads=kvh, device=ctx.dev) for layer in range(nd)]
    caches = [physical[layer % nd] for layer in range(geo.num_layers)]
    torch.cuda.synchronize()
    with tempfile.TemporaryDirectory() as d:
        m = W.b200_method(w, caches, W.write_stats_file(w, d), tp_size=ctx.world, tp_group=ctx.group,
                          tp_rank=ctx.rank, device=ctx.dev)
    reqs = W.b200_requests(w, device=ctx.dev)
    flusher = L2Flush(ctx.dev) if flush else None
    for _ in range(warmup):
        m.compress_many(reqs)
    m.check_device_errors()
    torch.cuda.synchronize()
    barrier(ctx)
    clk = None
    sampler = ClockSampler(ctx.local) if clocks else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    barrier(ctx)
    if flusher is None:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            m.compress_many(reqs)
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / steps
    else:  # inputs fit in L2: time each step alone, after a flush
        evs = []
        for g0 in range(0, steps, QUEUED):
            host_ahead()
            for _ in range(min(QUEUED, steps - g0)):
                flusher()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                m.compress_many(reqs)
                b.record()
                evs.append((a, b))
        torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    barrier(ctx)
    if sampler:
        clk = sampler.stop()
    m.check_device_errors()
    ms = max_over_ranks(ctx, ms)

    # per-stage breakdown: a separate, instrumented pass (stage events cost host time),
    # started together on all ranks so the first sync does not absorb their skew
    timer = StageTimer()
    torch.cuda.synchronize()
    barrier(ctx)
    m.profiler = timer
    timer.active = True
    for k in range(max(3, min(steps, 20))):
        if flusher:
            if k % QUEUED == 0:
                host_ahead()
            flusher()
        timer.new_step()
        m.compress_many(reqs)
    torch.cuda.synchronize()
    timer.active = False
    m.profiler = None
    barrier(ctx)
    stages = timer.stage_ms()
    tp_split = timer.exchange_us()

    # end to end through the public API with host buffers: every step copies its
    # block tables from pinned host memory into the provider's persistent
    # device buffer (H2D) and reads its staged commit rows/offsets back into
    # pinned host memory (D2H).  Steps are issued back to back as a serving
    # host does: the host waits for step k-1's read-back after issuing step k
    # (double-buffered outputs), and for the last one at the end of the region.
    e2e_steps = max(1, min(steps, 50))
    host_src = [torch.tensor(w.src_tables[i], dtype=torch.long) for i in w.compressed()]
    host_dst = [torch.tensor(w.dst_tables[i], dtype=torch.long) for i in w.compressed()]
    flat = torch.cat(host_src + host_dst).pin_memory()
    sizes = [t.numel() for t in host_src + host_dst]
    R = len(host_src)
    out_rows = [torch.empty((R, -(-w.options.kv_budget // 128)), dtype=torch.long).pin_memory() for _ in range(2)]
    out_off = [torch.empty(R, dtype=torch.long).pin_memory() for _ in range(2)]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    dflat = torch.empty_like(flat, device=ctx.dev)
    parts = torch.split(dflat, sizes)
    step_reqs = [replace(r, source_block_ids_device=parts[j], destination_block_ids_device=parts[R + j])
                 for j, r in enumerate(reqs)]
    checked = []

    def e2e_step(k: int, wait_previous: bool = True):
        b = k % 2
        dflat.copy_(flat, non_blocking=True)
        m.compress_many(step_reqs, stage_commit=True)
        out_rows[b].copy_(m.staged_block_rows, non_blocking=True)
        out_off[b].copy_(m.staged_offsets, non_blocking=True)
        done[b].record()
        if wait_previous and k > 0:
            done[(k - 1) % 2].synchronize()  # step k-1's result is on the host
            checked.append(int(out_off[(k - 1) % 2][0]))

    e2e_step(0, wait_previous=False)
    torch.cuda.synchronize()
    barrier(ctx)
    if flusher is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for k in range(e2e_steps):
            e2e_step(k)
        done[(e2e_steps - 1) % 2].synchronize()
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
    else:  # small inputs: one step at a time after an L2 flush
        tot = 0.0
        for k in range(e2e_steps):
            flusher()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            e2e_step(k, wait_previous=False)
            done[k % 2].synchronize()
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
        e2e_ms = tot / e2e_steps
    if checked and any(c != checked[0] for c in checked):
        raise SystemExit("staged commit offsets changed between identical steps")
    barrier(ctx)
    e2e_ms = max_over_ranks(ctx, e2e_ms)
    m.check_device_errors()
    # staged metadata: 6R+2 int64 and 2R+1 int32 words, copied as int64 words
    h2d = flat.numel() * 8 + (6 * R + 2 + (2 * R + 2) // 2) * 8
    d2h = out_rows[0].numel() * 8 + out_off[0].numel() * 8

    res = {"ms": ms, "e2e_ms": e2e_ms, "stages": stages, "clocks": clk, "h2d": h2d, "d2h": d2h, "kvh": kvh,
           "tp_sync_mode": m.tp_sync_mode, "parity": None, "cpu_baseline": None, "tp_split": tp_split}
    if check:
        s = collect_sample(ctx, w, m, physical, nd)
        if ctx.rank == 0:
            try:
                res["parity"] = parity_check(ctx, w, s)
            except Exception as exc:  # report, do not hide the line
                res["parity"] = {"ok": False, "error": f"{type(exc).__name__}: {exc}"}
            if cpu and ctx.world == 1:
                res["cpu_baseline"] = cpu_baseline(w, s)
        del s
        barrier(ctx)
    release(ctx, m)
    del m, caches, physical, reqs, step_reqs, parts, dflat
    gc.collect()
    torch.cuda.empty_cache()
    return res


def summarize(w: W.Workload, res: dict, world: int, nd: int) -> dict:
    """The JSON fields of one measured workload."""
    peak, peak_kind = peaks()
    tokens = w.total_compressed_tokens()
    ab = algorithmic_bytes(w, res["kvh"])
    st = res["stages"]
    step_bytes = sum(ab.values())
    ms = res["ms"]
    out = {
        "value": tokens / (ms * 1e-3), "unit": UNIT, "per_gpu": tokens / (ms * 1e-3) / world, "ms_per_step": ms,
        "config": config_dict(w, world, nd),
        "step_roofline": {"achieved": step_bytes / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                          "frac": step_bytes / (ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": step_bytes,
                          "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
        "stages_ms": st,
        "e2e": {"value": tokens / (res["e2e_ms"] * 1e-3), "unit": UNIT, "h2d_bytes_per_step": res["h2d"],
                "d2h_bytes_per_step": res["d2h"], "ms_per_step": res["e2e_ms"],
                "path": "TriAttentionMethod.compress_many(stage_commit=True) per step: pinned H2D block tables, "
                        "staged block rows/offsets read back D2H into pinned memory; steps issued back to back, "
                        "the host waits for each step's read-back one step later (double-buffered)"},
        "parity": res["parity"],
    }
    for name, key in (("compact", "compact"), ("score", "score")):
        t = st.get(name)
        if t:
            gbs = ab[key] / (t * 1e-3) / 1e9
            out[f"{name}_kernel"] = {"achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                                     "algorithmic_bytes": ab[key], "ms": t}
    if world > 1:
        out["tp_sync_us"] = st.get("tp_sync", 0.0) * 1e3
        out["tp_sync_path"] = res["tp_sync_mode"]
        if res.get("tp_split"):
            out["tp_sync_split"] = res["tp_split"]
    if res["cpu_baseline"]:
        out["cpu_baseline"] = {k: v for k, v in res["cpu_baseline"].items() if k != "seconds"}
    return out


def calib_case(ctx: Ctx, layers: int, cpu: bool = True) -> dict:
    """Config 3: calibration reduction of 64 x 8192 pre-RoPE queries (40 heads x 128) per layer."""
    from vllm_ascend_kvcompress.methods.triattention import kernels as K

    heads, hd, rot = 40, 128, 128
    n_seq, seq_len = 64, 8192
    n_tok = n_seq * seq_len
    need = K.calibration_workspace_doubles(n_tok, heads, hd, rot)
    ws = torch.empty(need, dtype=torch.float64, device=ctx.dev)
    z = lambda: torch.zeros(heads, rot // 2, dtype=torch.float64, device=ctx.dev)
    total_ms, worst = 0.0, 0.0
    cpu_line = None
    for layer in range(layers):
        q = W.calibration_queries(layer, n_seq, seq_len, heads, hd, device=ctx.dev)
        re, im, ab = z(), z(), z()
        for rep in range(4):  # three warm-up passes of layer 0, then the timed pass
            re.zero_(); im.zero_(); ab.zero_()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            K.calibration_accumulate(q, heads, hd, rot, re, im, ab, None, ws)
            b.record()
            torch.cuda.synchronize()
            if layer > 0:
                break
        total_ms += a.elapsed_time(b)
        if layer == 0:  # parity against an fp64 reduction of the same tensor
            v = q.view(-1, heads, hd).double()
            ref = (v[..., :rot // 2].sum(0), v[..., rot // 2:rot].sum(0),
                   torch.sqrt(v[..., :rot // 2].square() + v[..., rot // 2:rot].square()).sum(0))
            mean_abs = v.abs().mean().item()
            for g, r in zip((re, im, ab), ref):
                worst = max(worst, ((g - r).abs().max() / n_tok).item() / max(r.abs().max().item() / n_tok, mean_abs))
            del v
            if cpu and ctx.rank == 0:
                cpu_line = calib_cpu_baseline(q[: n_tok // 8].cpu(), heads, hd, rot)
        del q
    tokens = layers * n_tok
    bytes_ = tokens * heads * hd * 2.0
    peak, kind = peaks()
    gbs = bytes_ / (total_ms * 1e-3) / 1e9
    out = {
        "metric": "calibration query tokens reduced/s (config 3)", "value": tokens / (total_ms * 1e-3),
        "unit": "tokens/s", "ms_per_step": total_ms / layers, "steps": layers,
        "config": {"workload": f"config3: calibration reduction, {layers} layer(s) x {n_seq} x {seq_len} tokens, "
                               f"{heads} heads x head_dim {hd}", "layers": layers, "tokens_per_layer": n_tok,
                   "l2": "inputs (5.4 GB per layer) exceed L2; no flush needed"},
        "roofline": {"bound": "hbm", "kernel": "kvc calibration partial + finalize", "achieved": gbs, "peak": peak,
                     "unit": "GB/s", "frac": gbs / peak, "traffic": None, "peak_source": kind},
        "parity": {"max_err_over_scale_vs_fp64": worst, "tolerance": 1e-4, "ok": worst <= 1e-4},
    }
    if cpu_line:
        out["cpu_baseline"] = cpu_line
    return out


def calib_cpu_baseline(q: torch.Tensor, heads: int, hd: int, rot: int, repeats: int = 5) -> dict:
    """The oracle's reduction (calibration.py:95-131 restated) on 1/8 of one layer's tokens."""
    from oracle import triattention_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    times = []
    for _ in range(repeats + 1):
        acc = O.CalibrationSums()
        t0 = time.perf_counter()
        acc.add(q, heads, hd, rot)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times[1:])
    return {"value": q.shape[0] / t, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"oracle CalibrationSums.add on {q.shape[0]} of one layer's 524288 query tokens "
                      f"(40 heads x 128), median of {repeats}"}


def other_cases(world: int) -> list[int]:
    return {1: [0, 2, 3, 4], 2: [2, 4]}.get(world, [4])


def b200_arm(args) -> None:
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        group = dist.group.WORLD
    ctx = Ctx(rank, world, local, dev, group)
    if args.config == 3:
        line = calib_case(ctx, args.layers)
        if rank == 0:
            line.update({"n_gpus": 1, "warmup": 3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                         "dtype": "f32", "data": "synthetic pre-RoPE queries q ~ N(mu_h, 1), mu_h ~ N(0, 0.5), BF16"})
            print(json.dumps(line), flush=True)
        return
    w = make_workload(args.config, args)
    nd = distinct_layers(args.config, args, w)
    small = sum(algorithmic_bytes(w, w.geometry.num_kv_heads).values()) < 4 * L2_BYTES
    res = measure(ctx, w, nd, args.steps, args.warmup, clocks=True, check=not args.no_check,
                  cpu=not args.no_cpu_baseline, flush=small)
    other = {}
    if not args.no_other_configs and args.config == 1 and args.seqs == 32 and args.layers == 48:
        o_steps, o_warm = max(3, min(args.steps, 20)), max(3, min(args.warmup, 5))
        for c in other_cases(world):
            t0 = time.perf_counter()
            if c == 3:
                if rank == 0:
                    other["config3"] = calib_case(ctx, 1, cpu=not args.no_cpu_baseline)
                barrier(ctx)
            else:
                wc = make_workload(c, args)
                ndc = distinct_layers(c, args, wc)
                smallc = sum(algorithmic_bytes(wc, wc.geometry.num_kv_heads).values()) < 4 * L2_BYTES
                rc = measure(ctx, wc, ndc, o_steps if not smallc else max(o_steps, 50), o_warm, check=not args.no_check,
                             cpu=not args.no_cpu_baseline, flush=smallc)
                if rank == 0:
                    other[wc.name] = summarize(wc, rc, world, ndc)
            if rank == 0 and f"config{c}" in other:
                other[f"config{c}"]["wall_s"] = time.perf_counter() - t0
    if rank == 0:
        s = summarize(w, res, world, nd)
        peak, peak_kind = peaks()
        ck = s.get("compact_kernel", {})
        traffic = None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.is_file() and args.config == 1 and args.seqs == 32 and args.layers == 48 and world == 1:
            traffic = json.loads(tf.read_text()).get("compact_kernel_bytes_per_launch_config1")
        # tables, prepare, score, head stats, normalise, the layer reduction (or
        # the peer exchange kernel), select, compact; with one scoring layer at
        # N = 1 normalisation writes the aggregate itself (no layer reduction)
        scoring_layers = -(-w.geometry.num_layers // w.options.score_layer_stride)
        launches_per_step = 7 if (world == 1 and scoring_layers == 1) else 8
        line = {
            "metric": METRIC, "value": s["value"], "unit": UNIT, "value_is": "aggregate over all GPUs",
            "per_gpu": s["per_gpu"], "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": s["ms_per_step"], "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) BF16 K/V, random calibration stats)",
            "config": s["config"],
            "roofline": {"bound": "hbm", "kernel": "kvc compact (paged K/V gather-copy, all layers)",
                         "achieved": ck.get("achieved"), "peak": peak, "unit": "GB/s", "frac": ck.get("frac"),
                         "traffic": traffic, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": ck.get("algorithmic_bytes")},
            "step_roofline": s["step_roofline"], "stages_ms": s["stages_ms"],
            "score_kernel": s.get("score_kernel"),
            "tp_sync_us": s.get("tp_sync_us"), "tp_sync_path": res["tp_sync_mode"] if world > 1 else "none",
            "tp_sync_split": s.get("tp_sync_split"),
            "e2e": s["e2e"], "gpu_launches": launches_per_step * args.steps, "clocks": res["clocks"],
            "parity": s["parity"],
        }
        if "cpu_baseline" in s:
            line["cpu_baseline"] = s["cpu_baseline"]
        if other:
            line["other_configs"] = other
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--stride", type=int, default=8, help="score_layer_stride (8 = default, 1 = every layer)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the in-run result check (profiling only)")
    ap.add_argument("--no-other-configs", action="store_true", help="headline workload only")
    ap.add_argument("--seqs", type=int, default=32, help="sequences (32 = config 1; smaller only for profiling)")
    ap.add_argument("--layers", type=int, default=48, help="layers (48 = config 1; smaller only for profiling)")
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 2, 3, 4],
                    help="benchmark-specification configuration (1 = the headline line)")
    ap.add_argument("--distinct-layers", type=int, default=0,
                    help="physical caches aliased round-robin onto the layers (0 = all distinct; config 4 uses 5)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
    else:
        b200_arm(args)


if __name__ == "__main__":
    main()

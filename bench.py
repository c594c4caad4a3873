"""Benchmark of the B200 TriAttention score -> select -> compact pass.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--stride 8|1]

Workload (N = 1): the Qwen2.5-14B-shaped ragged batch of the benchmark
specification (config 1): 48 layers, 40 query / 8 KV heads, head_dim 128, RoPE
theta 1e6, BF16 K/V ~ N(0, 1), 128-token pages placed by a seeded permutation,
32 sequences of U[4096, 32768] tokens (seed 1), kv_budget 4608, recompute
window 128, V3 policy (prefix 128, recent 512, 8 segments), mean/mean
aggregation, score_layer_stride 8.  One step = one score + select + compact
pass over every compressed sequence and every layer.  Inputs (~145 GB of K/V)
are far larger than L2, so no flush is needed between steps.

N > 1 (torchrun, one process per GPU): the same batch with the 8 KV heads
sharded over N tensor-parallel ranks; every step issues one NCCL MAX
all-reduce of all per-layer score rows (strong scaling: total work fixed).

--impl reference times the CPU oracle (a restatement of the reference's own
torch CPU path) on a bounded sample of the same workload, with all host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "vllm-ascend-kvcompress-hust_b200"))

import torch  # noqa: E402

import kvc_workloads as W  # noqa: E402

METRIC = "KV tokens scored+compacted/s per GPU & % HBM roofline; TP score-sync µs at 2/4/8"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


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
# CPU baseline (oracle restatement of the reference's torch CPU path)
# ---------------------------------------------------------------------------


def cpu_sample_workload(w: W.Workload, seq: int) -> W.Workload:
    """One sequence of ``w`` on a minimal block pool (same geometry and options)."""
    return W.place_blocks(W.Workload(w.name + "-cpu-sample", w.geometry, w.options, [w.lengths[seq]], seed=w.seed))


def run_cpu_sample(w: W.Workload, seq: int, distinct_layers: int = 8, repeats: int = 1) -> tuple[float, dict]:
    """Time the oracle on one sequence with all layers; returns (tokens/s, description)."""
    from oracle import triattention_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sw = cpu_sample_workload(w, seq)
    geo = sw.geometry
    distinct = [W.kv_pages(sw, layer) for layer in range(distinct_layers)]
    caches = [distinct[i % distinct_layers] for i in range(geo.num_layers)]  # layer aliasing (same work)
    stats_one = O.stats_from_payload(W.calibration_payload(geo, w.seed), geo.num_kv_heads, geo.group,
                                     geo.rotary_dim, range(geo.num_layers))
    o = sw.options
    opts = O.OracleOptions(kv_budget=o.kv_budget, protected_prefix_window=o.protected_prefix_window,
                           protected_recent_window=o.protected_recent_window, position_segments=o.position_segments,
                           position_policy=o.position_policy, score_chunk_size=o.score_chunk_size,
                           score_layer_stride=o.score_layer_stride)
    offs = O.geometric_offsets(o.max_model_len)
    req = O.OracleRequest(sw.lengths[0], sw.lengths[0], torch.tensor(sw.src_tables[0]), torch.tensor(sw.dst_tables[0]))
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        _, keep = O.select_request([c[0] for c in caches], stats_one, req, opts, offs)
        for kc, vc in caches:
            O.materialize(kc, vc, req.src_blocks, req.dst_blocks, keep)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    desc = (f"oracle (torch CPU restatement of the reference path) on 1 sequence of {sw.lengths[0]} tokens, "
            f"all {geo.num_layers} layers (aliased onto {distinct_layers} distinct caches), "
            f"stride {o.score_layer_stride}, median of {repeats}")
    return sw.lengths[0] / t, {"threads": threads, "seconds": t, "sample": desc}


def reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    w = make_workload(args)
    seq = sorted(w.compressed(), key=lambda i: w.lengths[i])[len(w.compressed()) // 2]  # median-length sequence
    budget_s = 150.0
    t0 = time.perf_counter()
    run_cpu_sample(w, seq)  # warm-up (one step)
    step_s = time.perf_counter() - t0
    steps = max(2, min(args.steps, int(budget_s / max(step_s, 1e-3))))
    value, info = run_cpu_sample(w, seq, repeats=steps)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": 1, "ms_per_step": info["seconds"] * 1e3, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) BF16 K/V, random calibration stats)",
        "config": config_dict(w, world, distinct_layers(args, w)),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": info["threads"], "kind": "port",
                         "sample": info["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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


def make_workload(args) -> W.Workload:
    if args.config == 0:
        return W.config0()
    if args.config == 2:
        return W.config2()
    if args.config == 4:
        return W.config4(num_seqs=args.seqs if args.seqs != 32 else 128, stride=args.stride)
    return W.config1(stride=args.stride, num_seqs=args.seqs, num_layers=args.layers)


def distinct_layers(args, w: W.Workload) -> int:
    if args.distinct_layers:
        return min(args.distinct_layers, w.geometry.num_layers)
    return 5 if args.config == 4 else w.geometry.num_layers


def config_dict(w: W.Workload, world: int, distinct: int | None = None) -> dict:
    o = w.options
    return {
        "workload": WORKLOAD_TEXT[w.name].format(layers=w.geometry.num_layers, seqs=len(w.lengths),
                                                 distinct=distinct or w.geometry.num_layers),
        "global_batch": len(w.lengths), "compressed_sequences": len(w.compressed()),
        "compressed_tokens": w.total_compressed_tokens(), "layers": w.geometry.num_layers,
        "score_layer_stride": o.score_layer_stride, "kv_budget": o.kv_budget,
        "parallelism": f"tp{world}" if world > 1 else "single",
        "l2": "inputs (>100 GB of K/V) exceed L2; no flush needed",
    }


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------


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
    w = make_workload(args)
    geo = w.geometry
    if geo.num_kv_heads % world:
        raise SystemExit(f"{geo.num_kv_heads} KV heads cannot be sharded over {world} ranks")
    kvh = geo.num_kv_heads // world
    nd = distinct_layers(args, w)
    physical = [W.kv_pages(w, layer * world + rank, kv_heads=kvh, device=dev) for layer in range(nd)]
    caches = [physical[layer % nd] for layer in range(geo.num_layers)]
    torch.cuda.synchronize()
    with tempfile.TemporaryDirectory() as d:
        m = W.b200_method(w, caches, W.write_stats_file(w, d), tp_size=world, tp_group=group, tp_rank=rank,
                          device=dev)
    reqs = W.b200_requests(w, device=dev)
    timer = StageTimer()

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    for _ in range(args.warmup):
        m.compress_many(reqs)
    m.check_device_errors()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    start.record()
    for _ in range(args.steps):
        m.compress_many(reqs)
    end.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    m.check_device_errors()
    # per-stage breakdown: a separate, instrumented pass (stage events cost host time),
    # started together on all ranks so the first sync does not absorb their skew
    torch.cuda.synchronize()
    barrier()
    m.profiler = timer
    timer.active = True
    for _ in range(max(3, min(args.steps, 20))):
        timer.new_step()
        m.compress_many(reqs)
    torch.cuda.synchronize()
    timer.active = False
    m.profiler = None
    barrier()
    ms = start.elapsed_time(end) / args.steps
    stages = timer.stage_ms()
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)

    # ---- end to end through the public API with host buffers ---------------
    e2e_steps = max(1, min(args.steps, 50))
    host_src = [torch.tensor(w.src_tables[i], dtype=torch.long).pin_memory() for i in w.compressed()]
    host_dst = [torch.tensor(w.dst_tables[i], dtype=torch.long).pin_memory() for i in w.compressed()]
    flat = torch.cat(host_src + host_dst).pin_memory()
    sizes = [t.numel() for t in host_src + host_dst]
    R = len(host_src)
    out_rows = torch.empty((R, -(-w.options.kv_budget // 128)), dtype=torch.long).pin_memory()
    out_off = torch.empty(R, dtype=torch.long).pin_memory()
    from dataclasses import replace

    # the requests reference a persistent device buffer that each step refills from
    # pinned host memory (one H2D copy per step), as a provider with fixed buffers would
    dflat = torch.empty_like(flat, device=dev)
    parts = torch.split(dflat, sizes)
    step_reqs = [replace(r, source_block_ids_device=parts[j], destination_block_ids_device=parts[R + j])
                 for j, r in enumerate(reqs)]

    def e2e_step():
        dflat.copy_(flat, non_blocking=True)
        m.compress_many(step_reqs, stage_commit=True)
        out_rows.copy_(m.staged_block_rows, non_blocking=True)
        out_off.copy_(m.staged_offsets, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t)
    # block tables + the method's staged metadata (6R+2 int64 and 2R+1 int32, copied as int64 words)
    h2d = flat.numel() * 8 + (6 * R + 2 + (2 * R + 2) // 2) * 8
    d2h = out_rows.numel() * 8 + out_off.numel() * 8

    if rank == 0:
        tokens = w.total_compressed_tokens()
        peak, peak_kind = peaks()
        ab = algorithmic_bytes(w, kvh)
        comp_ms = stages.get("compact", float("nan"))
        score_ms = stages.get("score", float("nan"))
        comp_gbs = ab["compact"] / (comp_ms * 1e-3) / 1e9
        score_gbs = ab["score"] / (score_ms * 1e-3) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.is_file() and args.config == 1 and args.seqs == 32 and args.layers == 48:
            traffic = json.loads(tf.read_text()).get("compact_kernel_bytes_per_launch_config1")
        # block-table gather, prepare, score, head_stats, normalize, then aggregate_rows (TP=1 / NCCL)
        # or the two exchange kernels (peer sync), select, compact
        launches_per_step = 9 if m.tp_sync_mode == "peer" else 8
        step_bytes = sum(ab.values())
        line = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) BF16 K/V, random calibration stats)",
            "config": config_dict(w, world, nd),
            "roofline": {"bound": "hbm", "kernel": "kvc compact (paged K/V gather-copy, all layers)",
                         "achieved": comp_gbs, "peak": peak, "unit": "GB/s", "frac": comp_gbs / peak,
                         "traffic": traffic, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": ab["compact"]},
            "step_roofline": {"achieved": step_bytes / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                              "frac": step_bytes / (ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": step_bytes},
            "stages_ms": stages,
            "score_kernel": {"achieved": score_gbs, "frac": score_gbs / peak, "algorithmic_bytes": ab["score"]},
            "tp_sync_us": stages.get("tp_sync", 0.0) * 1e3 if world > 1 else None,
            "tp_sync_path": m.tp_sync_mode,
            "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "path": "TriAttentionMethod.compress_many(stage_commit=True): pinned H2D block tables, "
                            "staged block rows/offsets read back"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu_baseline:
            seq = sorted(w.compressed(), key=lambda i: w.lengths[i])[len(w.compressed()) // 2]
            v, info = run_cpu_sample(w, seq, distinct_layers=min(8, geo.num_layers))
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": info["threads"], "kind": "port",
                                    "sample": info["sample"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def calib_arm(args) -> None:
    """Config 3: calibration reduction of 48 layers x 64 x 8192 pre-RoPE queries (40 heads x 128)."""
    from vllm_ascend_kvcompress.methods.triattention import kernels as K

    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    heads, hd, rot = 40, 128, 128
    n_seq, seq_len = 64, 8192
    layers = args.layers if args.layers != 48 else 48
    n_tok = n_seq * seq_len
    need = K.calibration_workspace_doubles(n_tok, heads, hd, rot)
    ws = torch.empty(need, dtype=torch.float64, device=dev)
    z = lambda: torch.zeros(heads, rot // 2, dtype=torch.float64, device=dev)
    total_ms, worst = 0.0, 0.0
    for layer in range(layers):
        q = W.calibration_queries(layer, n_seq, seq_len, heads, hd, device=dev)
        re, im, ab = z(), z(), z()
        for _ in range(2):  # warm-up pass (layer 0) then the timed pass
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
        del q
    tokens = layers * n_tok
    bytes_ = tokens * heads * hd * 2.0
    peak, kind = peaks()
    gbs = bytes_ / (total_ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": "calibration query tokens reduced/s (config 3)", "value": tokens / (total_ms * 1e-3),
        "unit": "tokens/s", "n_gpus": 1, "steps": layers, "warmup": 1, "ms_per_step": total_ms / layers,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic pre-RoPE queries q ~ N(mu_h, 1), mu_h ~ N(0, 0.5), BF16",
        "config": {"workload": f"config3: calibration reduction, {layers} layers x {n_seq} x {seq_len} tokens, "
                               f"{heads} heads x head_dim {hd}", "layers": layers, "tokens_per_layer": n_tok},
        "roofline": {"bound": "hbm", "kernel": "kvc calibration partial + finalize", "achieved": gbs, "peak": peak,
                     "unit": "GB/s", "frac": gbs / peak, "traffic": None, "peak_source": kind},
        "parity_max_rel_err_vs_fp64": worst,
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--stride", type=int, default=8, help="score_layer_stride (8 = default, 1 = every layer)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    elif args.config == 3:
        calib_arm(args)
    else:
        b200_arm(args)


if __name__ == "__main__":
    main()

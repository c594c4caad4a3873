"""Seeded synthetic workloads for the score -> select -> compact path.

Shapes, sizes and value distributions follow the five configurations of the
benchmark specification (no public dataset is involved: keys/values are
N(0, 1) BF16 draws and calibration statistics are random with the stated
amplitude/phase laws).  This module is torch-only so that the golden-vector
script (which imports the reference plugin) and this repository's tests and
bench can share it without importing either plugin package.

Determinism: every random draw uses its own ``torch.Generator`` seeded from the
workload seed plus a fixed per-item salt, so CPU draws are identical on every
machine with the same torch build.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

BLOCK = 128
SALT_KV = 0
SALT_TABLE = 1000
SALT_STATS = 2000
SALT_LENGTHS = 3000


@dataclass(frozen=True)
class Geometry:
    num_layers: int          # materialised full-attention layers (N)
    num_kv_heads: int        # global KV heads
    num_q_heads: int         # global query heads
    head_dim: int
    rotary_dim: int
    rope_theta: float
    model_type: str = "qwen2"

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads


@dataclass(frozen=True)
class Options:
    kv_budget: int
    recompute_window: int = 128
    protected_prefix_window: int = 0
    protected_recent_window: int = 128
    position_segments: int = 8
    position_policy: str = "v3"
    score_aggregation: str = "mean"
    layer_aggregation: str = "mean"
    score_chunk_size: int = 8192
    score_layer_stride: int = 8
    max_model_len: int = 65536

    def method_config(self, stats_path: str) -> dict:
        return {
            "stats_path": stats_path,
            "auto_calibrate": False,
            "kv_budget": self.kv_budget,
            "recompute_window": self.recompute_window,
            "position_policy": self.position_policy,
            "protected_prefix_window": self.protected_prefix_window,
            "protected_recent_window": self.protected_recent_window,
            "position_segments": self.position_segments,
            "score_aggregation": self.score_aggregation,
            "layer_aggregation": self.layer_aggregation,
            "score_chunk_size": self.score_chunk_size,
            "score_layer_stride": self.score_layer_stride,
        }


@dataclass
class Workload:
    name: str
    geometry: Geometry
    options: Options
    lengths: list[int]                 # physical = semantic tokens per sequence
    seed: int
    cache_blocks_per_page: int = 1     # scheduler page / 128-token kernel block
    pool_pages: int | None = None      # kernel blocks in the shuffled source pool
    src_tables: list[list[int]] = field(default_factory=list)   # kernel block ids (expanded)
    dst_tables: list[list[int]] = field(default_factory=list)
    src_pages: list[list[int]] = field(default_factory=list)    # scheduler page ids (unexpanded)
    dst_pages: list[list[int]] = field(default_factory=list)
    num_blocks: int = 0

    @property
    def threshold(self) -> int:
        return self.options.kv_budget + self.options.recompute_window

    def compressed(self) -> list[int]:
        """Indices of sequences that reach the compression threshold."""
        return [i for i, t in enumerate(self.lengths) if t >= self.threshold]

    def total_compressed_tokens(self) -> int:
        return sum(self.lengths[i] for i in self.compressed())


def _pages(tokens: int, per_page: int) -> int:
    return (tokens + BLOCK * per_page - 1) // (BLOCK * per_page)


def place_blocks(w: Workload) -> Workload:
    """Source block tables from a seeded permutation of the pool; fresh dest blocks.

    Scheduler pages of ``cache_blocks_per_page`` kernel blocks are permuted and
    each expanded into consecutive kernel blocks (the provider's page expansion).
    Destination pages are fresh ids beyond the pool.
    """
    per = w.cache_blocks_per_page
    need = [_pages(t, per) for t in w.lengths]
    pool = w.pool_pages if w.pool_pages is not None else sum(need) * per
    pool_pages = pool // per
    if sum(need) > pool_pages:
        raise ValueError("pool too small for the sequences")
    g = torch.Generator().manual_seed(w.seed + SALT_TABLE)
    perm = torch.randperm(pool_pages, generator=g).tolist()
    src, src_pages, pos = [], [], 0
    for n in need:
        pages = perm[pos:pos + n]
        pos += n
        src_pages.append(pages)
        src.append([p * per + j for p in pages for j in range(per)])
    dst_pages_per_req = _pages(w.options.kv_budget, per)
    nxt = pool_pages
    dst, dst_pages = [], []
    for i in range(len(w.lengths)):
        if i in w.compressed():
            pages = list(range(nxt, nxt + dst_pages_per_req))
            nxt += dst_pages_per_req
            dst_pages.append(pages)
            dst.append([p * per + j for p in pages for j in range(per)])
        else:
            dst_pages.append([])
            dst.append([])
    w.src_tables, w.dst_tables, w.num_blocks = src, dst, nxt * per
    w.src_pages, w.dst_pages = src_pages, dst_pages
    return w


def calibration_payload(geo: Geometry, seed: int, layer_indices: list[int] | None = None) -> dict:
    """Schema-3 ``layer_stats`` payload with the benchmark's random statistics.

    Per query head and frequency pair: complex mean query with amplitude
    U(0.5, 2) and phase U(-pi, pi); mean |q| U(0.5, 2); freq_scale_sq = 1;
    inv_freq = theta^(-2i/rot); partial RoPE adds q_pass_mean ~ N(0, 0.1^2).
    """
    g = torch.Generator().manual_seed(seed + SALT_STATS)
    f = geo.rotary_dim // 2
    p = geo.head_dim - geo.rotary_dim
    layers = layer_indices if layer_indices is not None else list(range(geo.num_layers))
    inv_freq = 1.0 / (geo.rope_theta ** (torch.arange(0, geo.rotary_dim, 2, dtype=torch.float32) / geo.rotary_dim))
    stats = {}
    for li in layers:
        amp = 0.5 + 1.5 * torch.rand(geo.num_q_heads, f, generator=g)
        phase = (torch.rand(geo.num_q_heads, f, generator=g) * 2 - 1) * math.pi
        entry = {
            "q_mean_real": (amp * torch.cos(phase)).contiguous(),
            "q_mean_imag": (amp * torch.sin(phase)).contiguous(),
            "q_abs_mean": (0.5 + 1.5 * torch.rand(geo.num_q_heads, f, generator=g)).contiguous(),
            "freq_scale_sq": torch.ones(geo.num_q_heads, f),
            "inv_freq": inv_freq.clone(),
        }
        if p:
            entry["q_pass_mean"] = (0.1 * torch.randn(geo.num_q_heads, p, generator=g)).contiguous()
        stats[str(li)] = entry
    meta = {
        "schema_version": 3,
        "model_type": geo.model_type,
        "num_layers": geo.num_layers if layer_indices is None else max(layers) + 1,
        "num_attention_heads": geo.num_q_heads,
        "num_kv_heads": geo.num_kv_heads,
        "head_dim": geo.head_dim,
        "rotary_dim": geo.rotary_dim,
        "rope_theta": geo.rope_theta,
        "rope_style": "half",
        "rope_type": "default",
    }
    if layer_indices is not None:
        meta["attention_layer_indices"] = list(layers)
    return {"metadata": meta, "layer_stats": stats}


def kv_pages(w: Workload, layer: int, kv_heads: int | None = None, device="cpu",
             dtype=torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor]:
    """K and V caches ``[num_blocks, 128, kvh, D]`` ~ N(0, 1) for one layer.

    On CPU the draw is seeded per (workload, layer); on CUDA a device generator
    with the same seed is used (values then differ from the CPU draw, which
    only matters for benchmarks, never for parity tests).
    """
    kvh = kv_heads if kv_heads is not None else w.geometry.num_kv_heads
    shape = (w.num_blocks, BLOCK, kvh, w.geometry.head_dim)
    g = torch.Generator(device=device).manual_seed(w.seed + SALT_KV + 7919 * layer)
    k = torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(dtype)
    v = torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(dtype)
    return k, v


def _uniform_lengths(n: int, lo: int, hi: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(seed + SALT_LENGTHS)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


def config0() -> Workload:
    """CPU-runnable reference op: 1 layer, kvh 8, G 5, D 128, 4 sequences."""
    geo = Geometry(1, 8, 40, 128, 128, 1e6)
    opts = Options(kv_budget=2048, protected_prefix_window=4, protected_recent_window=128,
                   score_layer_stride=1)
    return place_blocks(Workload("config0", geo, opts, [1000, 2500, 4096, 6000], seed=0, pool_pages=128))


def config1(stride: int = 8, num_seqs: int = 32, num_layers: int = 48) -> Workload:
    """Qwen2.5-14B-shaped ragged batch: 48 layers, 40/8 heads, D 128, B 4608.

    ``num_seqs``/``num_layers`` shrink it for profiling captures only.
    """
    geo = Geometry(num_layers, 8, 40, 128, 128, 1e6)
    opts = Options(kv_budget=4608, recompute_window=128, protected_prefix_window=128,
                   protected_recent_window=512, score_layer_stride=stride)
    return place_blocks(Workload("config1", geo, opts, _uniform_lengths(num_seqs, 4096, 32768, 1), seed=1))


def config2(stride: int = 2) -> Workload:
    """Qwen3.5-35B-A3B-shaped hybrid (full-attention layers only), per-TP-rank view.

    10 full-attention layers, 16 query / 2 KV heads globally (TP=2 -> 1 local
    KV head, G 8), D 256 with partial RoPE over 64 dims, 2048-token logical
    pages expanded into 16 kernel blocks, B 4608.
    """
    geo = Geometry(10, 2, 16, 256, 64, 1e7, model_type="qwen3_5_moe_text")
    opts = Options(kv_budget=4608, recompute_window=1024, protected_prefix_window=128,
                   protected_recent_window=512, score_layer_stride=stride)
    return place_blocks(Workload("config2", geo, opts, _uniform_lengths(16, 8192, 53248, 2), seed=2,
                                 cache_blocks_per_page=16))


def config4(num_seqs: int = 128, stride: int = 8) -> Workload:
    """TP scaling sweep: config-1 heads, 128 sequences of U[2k, 64k] tokens."""
    geo = Geometry(48, 8, 40, 128, 128, 1e6)
    opts = Options(kv_budget=4608, recompute_window=128, protected_prefix_window=128,
                   protected_recent_window=512, score_layer_stride=stride)
    return place_blocks(Workload("config4", geo, opts, _uniform_lengths(num_seqs, 2048, 65536, 4), seed=4))


def calibration_queries(layer: int, n_seq: int, seq_len: int, heads: int, head_dim: int,
                        seed: int = 3, device="cpu") -> torch.Tensor:
    """Config 3: pre-RoPE prefill queries ``[n_seq*seq_len, heads*head_dim]`` BF16.

    q ~ N(mu_h, 1) with a fixed per-head offset mu_h ~ N(0, 0.5) (seeded per
    layer).  The reduction parity is defined on un-rotated queries, as the
    stats builder captures them before RoPE.
    """
    g = torch.Generator().manual_seed(seed * 100003 + layer)
    mu = 0.5 * torch.randn(heads, generator=g)
    gd = torch.Generator(device=device).manual_seed(seed * 100003 + layer + 1)
    q = torch.randn(n_seq * seq_len, heads, head_dim, generator=gd, device=device, dtype=torch.float32)
    q += mu.to(device).view(1, heads, 1)
    return q.to(torch.bfloat16).reshape(n_seq * seq_len, heads * head_dim)


def golden_calibration_inputs() -> list[tuple[str, int, int, int, list[torch.Tensor]]]:
    """Seeded pre-RoPE query batches of the calibration golden cases.

    (name, heads, head_dim, rotary_dim, [q per call]); one generator drives
    both cases in order, so the draws are reproducible without storing them.
    """
    g = torch.Generator().manual_seed(11)
    out = []
    for name, heads, hd, rot in (("calib_full", 4, 64, 64), ("calib_partial", 4, 64, 32)):
        calls = [(torch.randn(n, heads * hd, generator=g) + 0.3).to(torch.bfloat16) for n in (300, 500, 77)]
        out.append((name, heads, hd, rot, calls))
    return out


def golden_selection_scores(cases: list) -> list[torch.Tensor]:
    """Scores of the selection golden cases: successive ``randperm`` draws after
    ``torch.manual_seed(28)`` (the reference test's recipe), one per case."""
    torch.manual_seed(28)
    return [torch.randperm(c[0], dtype=torch.long).float() for c in cases]


# ---------------------------------------------------------------------------
# binding helpers for this repository's B200 package (imported lazily so the
# golden script, which imports the reference package of the same name, never
# touches them)
# ---------------------------------------------------------------------------


def layer_name(i: int) -> str:
    return f"model.layers.{i}.self_attn.attn"


def b200_method(w: Workload, caches, stats_path: str, *, tp_size: int = 1, tp_group=None, tp_rank=None,
                device="cuda", options: Options | None = None, geometry: Geometry | None = None):
    """Bind this package's TriAttentionMethod to ``caches`` [(k, v) per layer]."""
    from types import SimpleNamespace

    from vllm_ascend_kvcompress.methods.base import LayerCache, ModelShape
    from vllm_ascend_kvcompress.methods.triattention.method import TriAttentionMethod

    geo = geometry or w.geometry
    opts = options or w.options
    shape = ModelShape(model_type=geo.model_type, num_layers=geo.num_layers, num_attention_heads=geo.num_q_heads,
                       num_kv_heads=geo.num_kv_heads, head_dim=geo.head_dim, rope_theta=geo.rope_theta,
                       has_rope_scaling=False,
                       rotary_dim=None if geo.rotary_dim == geo.head_dim else geo.rotary_dim)
    vcfg = SimpleNamespace(parallel_config=SimpleNamespace(tensor_parallel_size=tp_size),
                           model_config=SimpleNamespace(max_model_len=opts.max_model_len),
                           speculative_config=None)
    m = TriAttentionMethod(opts.method_config(stats_path), vcfg, shape)
    runner = SimpleNamespace(device=torch.device(device), kvc_tp_group=tp_group, kvc_tp_rank=tp_rank)
    layers = tuple(LayerCache(name=layer_name(i), layer_index=i, k_cache=k, v_cache=v)
                   for i, (k, v) in enumerate(caches))
    m.bind_model_runner(runner, layers)
    return m


def b200_requests(w: Workload, device="cuda", indices: list[int] | None = None, pages: bool = False):
    """CompressionRequest objects of the workload's compressed sequences.

    ``pages``: the device tables hold scheduler page ids (for
    ``compress_many(..., cache_blocks_per_page=w.cache_blocks_per_page)``)
    instead of kernel block ids.
    """
    from vllm_ascend_kvcompress.methods.base import CompressionRequest

    src_t, dst_t = (w.src_pages, w.dst_pages) if pages else (w.src_tables, w.dst_tables)
    out = []
    for i in (indices if indices is not None else w.compressed()):
        out.append(CompressionRequest(
            request_id=f"r{i}", semantic_num_tokens=w.lengths[i], physical_num_tokens=w.lengths[i],
            source_block_ids=(tuple(w.src_pages[i]),), destination_block_ids=(tuple(w.dst_pages[i]),),
            source_block_ids_device=torch.tensor(src_t[i], dtype=torch.long, device=device),
            destination_block_ids_device=torch.tensor(dst_t[i], dtype=torch.long, device=device)))
    return out


def write_stats_file(w: Workload, directory) -> str:
    from pathlib import Path

    path = Path(directory) / f"{w.name}-stats.pt"
    torch.save(calibration_payload(w.geometry, w.seed), path)
    return str(path)

"""The bench's algorithmic byte model restates the per-step formula of the
benchmark specification: sum over compressed requests of
L_s*T*kvh*D*2 (K read for scoring) + N*B*kvh*D*2*2*2 (kept K and V rows read
and written), plus L_s*T*4 + B*8 (score rows and indices)."""

from __future__ import annotations

import bench
import kvc_workloads as W


def _formula(w: W.Workload, kvh: int) -> float:
    g, o = w.geometry, w.options
    ls = -(-g.num_layers // o.score_layer_stride)
    total = 0.0
    for i in w.compressed():
        t = w.lengths[i]
        total += ls * t * kvh * g.head_dim * 2 + g.num_layers * o.kv_budget * kvh * g.head_dim * 2 * 2 * 2
        total += ls * t * 4 + o.kv_budget * 8
    return total


def test_config0_bytes_match_the_specification():
    w = W.config0()
    ab = bench.algorithmic_bytes(w, w.geometry.num_kv_heads)
    # 3 compressed requests of 2500 + 4096 + 6000 tokens, 1 layer, kvh 8, D 128, B 2048
    assert w.total_compressed_tokens() == 12596
    assert ab["score"] == 12596 * 2048 + 12596 * 4
    assert ab["compact"] == 3 * 2048 * 2048 * 4
    # the specification's formula plus the selection's read of the final score row (T x 4 B)
    assert sum(ab.values()) == _formula(w, 8) + 12596 * 4


def test_byte_model_scales_with_tensor_parallel_shards():
    w = W.config1(stride=8, num_seqs=4, num_layers=8)
    full = bench.algorithmic_bytes(w, 8)
    shard = bench.algorithmic_bytes(w, 1)
    T = w.total_compressed_tokens()
    ls = -(-8 // 8)
    assert full["compact"] == 8 * shard["compact"]
    assert full["score"] - ls * T * 4 == 8 * (shard["score"] - ls * T * 4)

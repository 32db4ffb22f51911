"""The measurement's arithmetic (bench.py) against the per-unit figures of
the hot path's measurement plan: the algorithmic bytes of a configuration-2
decode step, the visible (query, key) pairs and FLOPs of the prefill
configurations, and the longest-first sharding of sequences over GPUs."""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_decode_step_bytes():
    """Per sequence 2·min(L,512)·256·2 + 2·L·512·2 bytes of f16 K/V, plus q
    read and output written (f32), the raw k/v read (f32) and the appended
    row (f16) of both layers; the seeded 64 contexts give the 304.2 MB that
    the bench line reports."""
    lens = [int(c) for c in bench.global_lengths(1)]
    assert len(lens) == 64 and min(lens) >= 1 and max(lens) <= 4096
    kv = sum(2 * min(c, 512) * 256 * 2 + 2 * c * 512 * 2 for c in lens)
    per_seq = sum(2 * 8 * hd * 4 + 2 * hd * 4 + 2 * hd * 2 for hd in (256, 512))
    sb = bench.step_bytes(lens)
    assert sb["total"] == kv + 64 * per_seq == sb["global"] + sb["local"]
    assert sb["total"] == 304_249_856
    assert sum(bench.kv_bytes(c) for c in lens) == kv


def test_prefill_pairs_and_flops():
    """Configuration 1 (628 tokens): 197,506 global and 190,720 sliding-window
    pairs, 66.40 GFLOP over 7 global and 28 local layers at 4·8·hd FLOPs per
    pair; configuration 3 (32,768 tokens): 536,887,296 pairs, 8.796 TFLOP."""
    g, l = bench.prefill_pairs(628, 0), bench.prefill_pairs(628, 512)
    assert (g, l) == (197_506, 190_720)
    flops = 7 * 4 * 8 * 512 * g + 28 * 4 * 8 * 256 * l
    assert round(flops / 1e9, 2) == 66.40
    t = 32768
    assert t * (t + 1) // 2 == 536_887_296
    assert round(4 * 8 * 512 * t * (t + 1) // 2 / 1e12, 3) == 8.796


def test_shards_cover_and_balance():
    """Every sequence on exactly one GPU, the same count on each, and the
    longest-first assignment within one sequence's bytes of balance."""
    for n in (2, 4, 8):
        lens = bench.global_lengths(n)
        parts = [bench.shard(lens, n, r) for r in range(n)]
        assert all(len(p) == len(lens) // n for p in parts)
        assert sorted(np.concatenate(parts).tolist()) == sorted(lens.tolist())
        loads = [sum(bench.kv_bytes(int(c)) for c in p) for p in parts]
        assert max(loads) - min(loads) <= max(bench.kv_bytes(int(c)) for c in lens)

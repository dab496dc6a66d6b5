"""Byte accounting behind bench.py's roofline figures (CPU only)."""
from __future__ import annotations

import bench
from dpuf_b200 import model as mdl


def test_expanded_bytes_match_the_gemm_layout():
    # per 128-row group and 32-column block: 4,096 B of s8 weights + 256 B of fp16 row scales
    s = mdl.QWEN3_8B
    q = 32 * 128 * 4352            # 4096 x 4096: 32 groups x 128 blocks
    kv = 8 * 128 * 4352            # 1024 x 4096
    gate = 96 * 128 * 4352         # 12288 x 4096
    down = 32 * 384 * 4352         # 4096 x 12288
    assert s.expanded_bytes_per_layer() == q + 2 * kv + q + 2 * gate + down
    # a row count that is not a multiple of 128 rounds up to whole groups (missing rows are zero)
    t = mdl.TINY_G3  # q 384x256: 3 groups x 8 blocks; k, v 128x256: 1 x 8; o 256x384: 2 x 12;
    #                   gate, up 512x256: 4 x 8; down 256x512: 2 x 16
    assert t.expanded_bytes_per_layer() == ((3 + 1 + 1) * 8 + 2 * 12 + 2 * 4 * 8 + 2 * 16) * 4352


def test_prefill_roofline_arithmetic():
    s = mdl.QWEN3_8B
    r = bench.prefill_roofline(s, 32, 0.01, 6545.9, "measured")
    # LM head: 16 + 2 * 128 * 144 = 36,880 B per tile, padded to 64
    assert r["bytes"] == s.layers * s.expanded_bytes_per_layer() + (s.vocab + 15) // 16 * 36928
    assert abs(r["frac"] - r["bytes"] / 0.01 / 1e9 / 6545.9) < 1e-4

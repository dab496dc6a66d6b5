"""Parity scenarios shared by the golden-fixture generator and the tests.

Each engine scenario is: a synthetic model shape and seed, environment knobs, a prompt and a
number of greedy decode steps (the reference CLI's run_turn_ex, dpuf-cli.c:2344-2420).
Golden outputs were produced by the reference engine built from its own sources
(oracle/build_ref.sh) and the reference packer; see make_golden.py.
"""
from __future__ import annotations

import dataclasses
import hashlib

import numpy as np


@dataclasses.dataclass(frozen=True)
class EngineScenario:
    name: str
    shape: str
    prompt_len: int
    n_decode: int
    env: tuple = ()
    norm_jitter: float = 0.0
    seed: int = 0
    all_logits: bool = False  # also record the prefill with only_last_logits = 0
    full_logits: bool = False  # store the full logit vectors (small vocab only)
    kv_type: int = 0  # DpufModelConfig.kv_type: 0 fp32 cache, 1 int8 cache with per-32 scales
    hybrid: bool = False  # every matrix in mode 13 or 14, as the reference's had4p-hybrid packing assigns


ENGINE_SCENARIOS = [
    EngineScenario("tiny_gqa", "tiny", 20, 12, norm_jitter=0.1, all_logits=True, full_logits=True),
    EngineScenario("tiny_mha_slab", "tiny-mha", 50, 8, env=(("DPUF_SWIGLU_DEADZONE", "0.02"),), norm_jitter=0.1),
    EngineScenario("tiny_keep_tiles", "tiny", 61, 9,
                   env=(("DPUF_PREFILL_KEEP_TILES", "12"), ("DPUF_GEN_KEEP_TILES", "14")), norm_jitter=0.1),
    EngineScenario("tiny_zone_a", "tiny-zone", 20, 16,
                   env=(("DPUF_EARLY_TILES", "300"), ("DPUF_EARLY_MARGIN", "0.05")), norm_jitter=0.1),
    EngineScenario("tiny_long", "tiny", 200, 60, seed=3),
    EngineScenario("qwen3_0_6b_pp32_tg32", "qwen3-0.6b", 32, 32),
    # Q8 KV cache (kv_type 1): pairs, a pair plus a lone head, lone heads only; odd and even
    # key counts (the pair path's odd last key)
    EngineScenario("tiny_q8", "tiny", 20, 12, norm_jitter=0.1, all_logits=True, full_logits=True, kv_type=1),
    EngineScenario("tiny_g3_q8", "tiny-g3", 33, 9, norm_jitter=0.1, seed=4, full_logits=True, kv_type=1),
    EngineScenario("tiny_mha_q8", "tiny-mha", 17, 8, norm_jitter=0.1, seed=2, kv_type=1),
    EngineScenario("qwen3_0_6b_q8", "qwen3-0.6b", 16, 8, kv_type=1),
    # fp32 KV cache past 2048 positions: a 2040-token prompt in 256-token chunks, then decode
    # steps whose attention reads up to 2052 keys
    EngineScenario("tiny_long_2k", "tiny-long", 2040, 12, norm_jitter=0.1, seed=5),
    # modes 13 / 14 as engine layers (had4p-hybrid: q, gate, up, odd-layer o and the embedding in
    # mode 13; k, v, down, even-layer o and the LM head in mode 14), also with pruned down tiles
    EngineScenario("tiny_hybrid", "tiny", 20, 12, norm_jitter=0.1, all_logits=True, full_logits=True, hybrid=True),
    EngineScenario("tiny_hybrid_keep", "tiny-mha", 37, 9, env=(("DPUF_PREFILL_KEEP_TILES", "12"),
                                                                ("DPUF_GEN_KEEP_TILES", "14")),
                   norm_jitter=0.1, seed=7, hybrid=True),
    # the Qwen3-0.6B shape as a hybrid model (tied mode-13 embedding as the LM head)
    EngineScenario("qwen3_0_6b_hybrid", "qwen3-0.6b", 32, 8, hybrid=True),
    # Zone A on a tied hybrid model: the LM head is the mode-13 embedding
    EngineScenario("tiny_zone_a_hybrid", "tiny-zone", 20, 16,
                   env=(("DPUF_EARLY_TILES", "300"), ("DPUF_EARLY_MARGIN", "0.05")), norm_jitter=0.1, seed=4,
                   hybrid=True),
]

# Packer cases: (rows, cols, tensor name used for the column signs, generator seed).
PACK_CASES = [
    (64, 64, "t0", 1),
    (72, 128, "blk.0.qkv_in", 2),
    (100, 256, "x", 3),
    (256, 1024, "blk.3.ffn_down.weight", 4),
    (1000, 512, "output.weight", 5),
    (4104, 192, "odd", 6),
]

# Standalone matmul cases: (pack case index, M, input kind).
MATMUL_CASES = [
    (3, 1, "normal"),
    (3, 7, "normal"),
    (4, 1, "sparse"),   # zero blocks exercise the xs == 0 skip
    (4, 50, "normal"),  # M >= 24: the reference's multi-slab path
    (5, 3, "normal"),   # ragged last tile (4104 rows)
]


# Modes 13 (QR_HAD4_ASYM) and 14 (QR_HAD6) standalone matmul: (rows, cols, mode, seed).  The
# blobs come from the reference packer (encode_tensor_qr_had4_asym / _had6) and are stored in
# had_asym.npz with the reference library's outputs; rows that are not a multiple of 16 give a
# ragged last tile (and a half-empty 8-row group).
HAD_CASES = [(72, 256, 13, 1), (100, 512, 14, 2), (256, 512, 13, 3), (264, 512, 14, 4)]
HAD_MATMUL = [(0, 1, "normal"), (0, 5, "normal"), (1, 1, "normal"), (1, 7, "normal"), (2, 1, "sparse"),
              (2, 13, "normal"), (3, 1, "normal"), (3, 6, "sparse")]


# forward_batch_ex with embeds_in (dpuf_engine.c:1658-1672): model shape, seed, rows, and the
# ids of the mixed call (-1: the row comes from embeds_in).
EMBEDS_CASE = ("tiny", 5, 12)
EMBEDS_MIXED_NEG = (2, 5, 11)


def embeds_input(rows: int, hidden: int) -> np.ndarray:
    return (np.random.default_rng(4242).standard_normal((rows, hidden)) * 0.05).astype(np.float32)


def deepstack_input(rows: int, hidden: int) -> list:
    """Three DeepStack row sets [rows][hidden] (the one-token call uses the first row of each)."""
    rng = np.random.default_rng(4343)
    return [(rng.standard_normal((rows, hidden)) * 0.02).astype(np.float32) for _ in range(3)]


MROPE_SECTION = (4, 6, 6)


def rope_positions(rows: int):
    """pos_t / pos_h / pos_w of the M-RoPE prefill: distinct for most rows, equal for row 0."""
    m = np.arange(rows, dtype=np.int32)
    return m.copy(), (m // 3).astype(np.int32), (m % 4).astype(np.int32)


def had_embed_ids(case_idx: int, rows: int) -> np.ndarray:
    """Row ids for the mode-13/14 embedding fixtures: the first and last rows (the last tile may
    be ragged) and seeded random rows."""
    rng = np.random.default_rng(900 + case_idx)
    return np.concatenate([[0, rows - 1], rng.integers(0, rows, 7)]).astype(np.int32)


def matmul_input(case_idx: int, M: int, kind: str, cols: int) -> np.ndarray:
    rng = np.random.default_rng(1000 + 17 * case_idx + M)
    x = rng.standard_normal((M, cols)).astype(np.float32)
    if kind == "sparse":
        x[:, : cols // 2] = 0.0
        x[:, cols // 2: cols // 2 + 32] *= np.float32(1e-6)
    return x


def logits_digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()[:32]


def blob_digest(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()

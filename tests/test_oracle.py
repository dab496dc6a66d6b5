"""The CPU oracle (oracle/dpuf_oracle.c) reproduces the reference's golden outputs bit for bit.

These pin the checker that the GPU parity tests compare against."""
import numpy as np
import pytest

import scenarios as sc
from _util import bitexact, golden_arrays, golden_engine, pack_case_blob, run_scenario
from oracle import oracle as orc


@pytest.mark.parametrize("ci,M,kind", sc.MATMUL_CASES)
def test_oracle_matmul_matches_reference(ci, M, kind):
    bv = pack_case_blob(ci)
    x = sc.matmul_input(ci, M, kind, bv.cols)
    got = orc.oracle_matmul(M, bv, x)
    assert bitexact(got, golden_arrays("matmul.npz")[f"matmul_{ci}_{M}_{kind}"])


@pytest.mark.parametrize("ci", [3, 4])
def test_oracle_embed_matches_reference(ci):
    g = golden_arrays("matmul.npz")
    bv = pack_case_blob(ci)
    ids = g[f"embed_{ci}_ids"]
    out = np.empty((len(ids), bv.cols), np.float32)
    orc.OracleEngine.lib_().orc_embed_mode12_f32(len(ids), bv.cols, ids.ctypes.data, bv.tiles.ctypes.data,
                                                 bv.tile_offsets.ctypes.data, bv.sign_bits.ctypes.data,
                                                 out.ctypes.data)
    assert bitexact(out, g[f"embed_{ci}"])


@pytest.mark.parametrize("ci,M,kind", sc.HAD_MATMUL)
def test_oracle_had_asym_matches_reference(ci, M, kind):
    """Modes 13 / 14: the restatement reproduces the reference library's outputs on blobs made
    by the reference packer (tests/golden/had_asym.npz)."""
    from dpuf_b200 import packer

    g = golden_arrays("had_asym.npz")
    rows, cols, mode, _ = sc.HAD_CASES[ci]
    bv = packer.BlobView(g[f"blob_{ci}"])
    assert (bv.mode, bv.rows, bv.cols) == (mode, rows, cols)
    x = sc.matmul_input(50 + ci, M, kind, cols)
    assert bitexact(orc.oracle_matmul_had(mode, M, bv, x), g[f"out_{ci}_{M}_{kind}"])


@pytest.mark.parametrize("ci", range(len(sc.HAD_CASES)))
def test_oracle_had_embed_matches_reference(ci):
    from dpuf_b200 import packer

    g = golden_arrays("had_asym.npz")
    rows, cols, mode, _ = sc.HAD_CASES[ci]
    bv = packer.BlobView(g[f"blob_{ci}"])
    assert bitexact(orc.oracle_embed_had(mode, bv, sc.had_embed_ids(ci, rows)), g[f"embed_{ci}"])


def test_swiglu_range_split_matches_reference_threads():
    lib = orc.OracleEngine.lib_()
    # I = 3072, M = 1 over 8 threads: every range is a multiple of 8 -> all vector
    assert all(lib.orc_swiglu_is_vector(i, 3072, 8) for i in range(0, 3072, 97))
    # M * I = 100 over 6 threads: ranges [0,16) [16,33) [33,50) ...; 17-element ranges end
    # with one scalar-tail element
    flags = [lib.orc_swiglu_is_vector(i, 100, 6) for i in range(100)]
    assert flags[:32] == [1] * 32 and flags[32] == 0 and flags[33:41] == [1] * 8 and flags[49] == 0


@pytest.mark.parametrize("scn", [s for s in sc.ENGINE_SCENARIOS if s.shape != "qwen3-0.6b"], ids=lambda s: s.name)
def test_oracle_engine_matches_reference(scn):
    g = golden_engine()[scn.name]
    rec, logits, _ = run_scenario(orc.OracleEngine, scn)
    assert rec["prompt"] == g["prompt"]
    assert rec["ids"] == g["ids"]
    assert rec["digests"] == g["digests"]
    if scn.all_logits:
        assert rec["prefill_all_digest"] == g["prefill_all_digest"]
    if scn.full_logits:
        assert bitexact(np.stack(logits), golden_arrays("engine_logits.npz")[scn.name])
    if "zone_exit" in g:
        za = max(256, int(dict(scn.env)["DPUF_EARLY_TILES"]))
        assert [bool(np.all(l[16 * za:] == np.float32(-1e9))) for l in logits] == g["zone_exit"]


@pytest.mark.slow
@pytest.mark.parametrize("scn", [s for s in sc.ENGINE_SCENARIOS if s.shape == "qwen3-0.6b"], ids=lambda s: s.name)
def test_oracle_qwen3_0_6b_matches_reference(scn):
    g = golden_engine()[scn.name]
    rec, _, _ = run_scenario(orc.OracleEngine, scn)
    assert rec["ids"] == g["ids"]
    assert rec["digests"] == g["digests"]


def test_zone_a_restatement():
    """Sequential top-2 of dpuf_engine.c:2101-2135: a repeated maximum is also the second place,
    margin <= 0 never exits, exit masks everything past the zone."""
    from oracle import oracle as orc

    lg = np.zeros(64, np.float32)
    lg[3] = 5.0
    lg[40] = 9.0  # outside a 2-tile zone (32 rows)
    ex, masked, b1, b2 = orc.zone_a(lg, 2, 1.0)
    assert ex and (b1, b2) == (5.0, 0.0)
    assert np.all(masked[32:] == np.float32(-1e9)) and masked[3] == 5.0
    lg[7] = 5.0
    assert not orc.zone_a(lg, 2, 1.0)[0]
    lg[7] = 0.0
    assert not orc.zone_a(lg, 2, 0.0)[0]


def test_q8_quantizer_restatement():
    """quantize_vec_q8_blk32 (dpuf_engine.c:751-781): scale = amax / 127, round half to even,
    a zero block gives scale 0 and zeros, an infinite element gives an infinite scale, zeros
    for its finite neighbours (x * 0) and -127 for itself (inf * 0 = NaN, which the x86
    conversion turns into INT32_MIN), and values saturate at +-127."""
    import ctypes

    lib = orc.OracleEngine.lib_()
    lib.orc_quantize_q8_blk32.argtypes = [ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    x = np.zeros(128, np.float32)
    x[32:64] = np.linspace(-1.0, 1.0, 32, dtype=np.float32)
    x[64:96] = 0.0
    x[64] = 127.0
    x[65:70] = [0.5, 1.5, 2.5, -0.5, -2.5]  # ties to even at inv = 1
    x[96:128] = 1.0
    x[100] = np.inf
    q = np.empty(128, np.int8)
    s = np.empty(4, np.float32)
    lib.orc_quantize_q8_blk32(128, x.ctypes.data, q.ctypes.data, s.ctypes.data)
    assert s[0] == 0.0 and np.all(q[:32] == 0)
    assert s[1] == np.float32(1.0) / np.float32(127.0) and q[32] == -127 and q[63] == 127
    assert s[2] == np.float32(1.0) and list(q[64:70]) == [127, 0, 2, 2, 0, -2]
    assert np.isinf(s[3]) and q[100] == -127 and np.all(np.delete(q[96:128], 4) == 0)

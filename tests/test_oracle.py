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
def test_oracle_qwen3_0_6b_matches_reference():
    scn = [s for s in sc.ENGINE_SCENARIOS if s.shape == "qwen3-0.6b"][0]
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

"""Modes 13 (QR_HAD4_ASYM) and 14 (QR_HAD6) standalone matmul on the GPU, through the reference's
exported signatures: bit-identical to the reference library's outputs on blobs made by the
reference packer (tests/golden/had_asym.npz), and to the oracle across token chunks."""
import ctypes

import numpy as np
import pytest

import scenarios as sc
from _util import bitexact, golden_arrays

pytestmark = pytest.mark.gpu

_SIG = [ctypes.c_int32] * 4 + [ctypes.c_void_p] * 5


@pytest.fixture(scope="module")
def lib():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dpuf_b200 import engine

    L = engine.cuda_lib()
    L.dpuf_matmul_qr_had4_asym_f32.argtypes = _SIG
    L.dpuf_matmul_qr_had6_f32.argtypes = _SIG
    return L


def _run(lib, mode, M, bv, x, rows=None, out=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = bv.rows if rows is None else rows
    out = np.empty((M, rows), np.float32) if out is None else out
    fn = lib.dpuf_matmul_qr_had4_asym_f32 if mode == 13 else lib.dpuf_matmul_qr_had6_f32
    fn(M, rows, bv.cols, bv.n_tiles, x.ctypes.data, bv.tiles.ctypes.data, bv.tile_offsets.ctypes.data,
       bv.sign_bits.ctypes.data, out.ctypes.data)
    return out


def _case(ci):
    from dpuf_b200 import packer

    g = golden_arrays("had_asym.npz")
    return g, packer.BlobView(g[f"blob_{ci}"]), sc.HAD_CASES[ci]


@pytest.mark.parametrize("ci,M,kind", sc.HAD_MATMUL)
def test_had_asym_matches_reference(lib, ci, M, kind):
    g, bv, (rows, cols, mode, _) = _case(ci)
    x = sc.matmul_input(50 + ci, M, kind, cols)
    assert bitexact(_run(lib, mode, M, bv, x), g[f"out_{ci}_{M}_{kind}"])


@pytest.mark.parametrize("ci", [2, 3])
def test_had_asym_token_chunks_match_oracle(lib, ci):
    """300 tokens: two prep + matmul chunks of the entry point."""
    from oracle import oracle as orc

    _, bv, (rows, cols, mode, _) = _case(ci)
    x = np.random.default_rng(ci).standard_normal((300, cols)).astype(np.float32)
    x[::7, :64] = 0.0  # zero blocks (block scale 0)
    assert bitexact(_run(lib, mode, 300, bv, x), orc.oracle_matmul_had(mode, 300, bv, x))


def test_had_asym_rejects_bad_descriptors(lib):
    from dpuf_b200 import engine

    _, bv, (rows, cols, mode, _) = _case(1)  # 100 rows: 7 tiles, the last one with 4 rows
    x = np.ones((1, cols), np.float32)
    sentinel = np.full((1, rows), 7.0, np.float32)
    # rows smaller than the tiles cover: the last tile would write past the output
    out = _run(lib, mode, 1, bv, x, rows=rows - 8, out=sentinel[:, :rows - 8].copy())
    assert np.all(out == 7.0) and "outside the matrix" in engine.last_error()
    lib.dpuf_matmul_qr_had6_f32(1, rows, cols - 32, bv.n_tiles, x.ctypes.data, bv.tiles.ctypes.data,
                                bv.tile_offsets.ctypes.data, bv.sign_bits.ctypes.data, sentinel.ctypes.data)
    assert np.all(sentinel == 7.0) and "descriptor" in engine.last_error()


def test_had_asym_timed_entry_point(lib):
    _, bv, (rows, cols, mode, _) = _case(2)
    lib.dpuf_cuda_had_asym_timed.argtypes = [ctypes.c_int32] * 5 + [ctypes.c_void_p] * 4 + [ctypes.c_int32] * 2 + \
        [ctypes.c_void_p]
    x = np.random.default_rng(0).standard_normal((4, cols)).astype(np.float32)
    ms = ctypes.c_float()
    assert lib.dpuf_cuda_had_asym_timed(mode, 4, rows, cols, bv.n_tiles, x.ctypes.data, bv.tiles.ctypes.data,
                                        bv.tile_offsets.ctypes.data, bv.sign_bits.ctypes.data, 2, 5,
                                        ctypes.byref(ms)) == 0
    assert ms.value > 0.0
    assert lib.dpuf_cuda_had_asym_timed(12, 4, rows, cols, bv.n_tiles, x.ctypes.data, bv.tiles.ctypes.data,
                                        bv.tile_offsets.ctypes.data, bv.sign_bits.ctypes.data, 2, 5,
                                        ctypes.byref(ms)) == -1


@pytest.mark.parametrize("ci", range(len(sc.HAD_CASES)))
def test_had_embed_matches_reference(lib, ci):
    g, bv, (rows, cols, mode, _) = _case(ci)
    ids = sc.had_embed_ids(ci, rows)
    fn = lib.dpuf_embed_qr_had4_asym_f32 if mode == 13 else lib.dpuf_embed_qr_had6_f32
    fn.argtypes = [ctypes.c_int32] * 2 + [ctypes.c_void_p] * 5
    out = np.empty((ids.size, cols), np.float32)
    fn(ids.size, cols, ids.ctypes.data, bv.tiles.ctypes.data, bv.tile_offsets.ctypes.data, bv.sign_bits.ctypes.data,
       out.ctypes.data)
    assert bitexact(out, g[f"embed_{ci}"])


def test_had_embed_rejects_rows_outside_tiles(lib):
    from dpuf_b200 import engine

    _, bv, (rows, cols, mode, _) = _case(1)  # 100 rows: the last tile holds rows 96..99
    lib.dpuf_embed_qr_had6_f32.argtypes = [ctypes.c_int32] * 2 + [ctypes.c_void_p] * 5
    for bad in (rows, -1):
        ids = np.array([3, bad], np.int32)
        out = np.full((2, cols), 7.0, np.float32)
        lib.dpuf_embed_qr_had6_f32(2, cols, ids.ctypes.data, bv.tiles.ctypes.data, bv.tile_offsets.ctypes.data,
                                   bv.sign_bits.ctypes.data, out.ctypes.data)
        assert np.all(out == 7.0) and engine.last_error(), bad


@pytest.mark.parametrize("mode", [13, 14])
@pytest.mark.parametrize("cols", [4096, 12288])
def test_had_rows_of_many_stages_match_oracle(lib, mode, cols):
    """Rows of 4,096 and 12,288 columns: the one-token kernel streams each 8-row group through
    its shared-memory ring in several stages (slots reused), the several-token kernel in many
    batches; both against the oracle (pinned to the reference's fixtures above)."""
    from dpuf_b200 import packer
    from oracle import oracle as orc

    h = packer.HadTiles(mode, 72, cols, seed=cols + mode)
    x = np.random.default_rng(cols + mode).standard_normal((3, cols)).astype(np.float32)
    x[:, 64:128] = 0.0  # a zero block (block scale 0)
    for M in (1, 3):
        assert bitexact(_run(lib, mode, M, h, x[:M]), orc.oracle_matmul_had(mode, M, h, x[:M])), M

"""Mode-12 packer: byte-exact against the reference packer (golden digests) and its helpers."""
import zlib

import numpy as np
import pytest

import scenarios as sc
from _util import golden_pack, pack_case_blob
from dpuf_b200 import packer


@pytest.mark.parametrize("i", range(len(sc.PACK_CASES)))
def test_blob_matches_reference_packer(i):
    g = golden_pack()[f"case{i}"]
    bv = pack_case_blob(i)
    assert sc.blob_digest(bv.blob) == g["sha256"]
    assert (bv.rows, bv.cols, bv.mode) == (g["rows"], g["cols"], 12)


def test_blob_view_fields():
    bv = pack_case_blob(5)  # 4104 rows: ragged last tile
    assert bv.n_tiles == (4104 + 15) // 16
    assert bv.tile_offsets[0] == 0
    last = bv.tiles[int(bv.tile_offsets[bv.n_tiles - 1]):]
    assert int(last[4]) | (int(last[5]) << 8) == 4104 - 16 * (bv.n_tiles - 1)
    assert len(bv.sign_bits) == bv.cols // 8


def test_tile_crc_matches_zlib():
    bv = pack_case_blob(3)
    n_blk = bv.cols // 32
    for t in (0, 7, bv.n_tiles - 1):
        tp = bv.tiles[int(bv.tile_offsets[t]):]
        body_len = 2 * n_blk * 144
        crc = int(tp[:4].view(np.uint32)[0])
        assert crc == (zlib.crc32(bytes(tp[16:16 + body_len])) & 0xFFFFFFFF)


def test_sign_bits_follow_reference_seeding():
    # seed = crc32(name) ^ 0x9E3779B9, one uint8 draw per column, little-endian bit packing
    bits = packer.sign_bits_for(128, "blk.0.qkv_in")
    rng = np.random.default_rng(zlib.crc32(b"blk.0.qkv_in") ^ 0x9E3779B9)
    flags = rng.integers(0, 2, size=128, dtype=np.uint8)
    assert np.array_equal(np.unpackbits(bits, bitorder="little"), flags)


def test_seed_names_shared_by_co_inputs():
    assert packer.hadamard_seed_name("blk.3.attn_k.weight") == "blk.3.qkv_in"
    assert packer.hadamard_seed_name("blk.3.ffn_up.weight") == "blk.3.mlp_in"
    assert packer.hadamard_seed_name("blk.3.ffn_down.weight") == "blk.3.ffn_down.weight"
    assert packer.hadamard_seed_name("output.weight") == "output.weight"


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-39, np.inf], dtype=np.float32)
    u = x.view(np.uint32)
    ref = ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)
    assert np.array_equal(packer.fp32_to_bf16(x), ref)


def test_generator_is_thread_count_independent():
    a = packer.gen_normal_bf16(7, 11, (333, 64), 0.02, n_threads=1)
    b = packer.gen_normal_bf16(7, 11, (333, 64), 0.02, n_threads=4)
    assert np.array_equal(a, b)
    f = (a.astype(np.uint32) << 16).view(np.float32)
    assert abs(float(f.std()) - 0.02) < 0.002


def test_rejects_bad_shapes():
    with pytest.raises(ValueError):
        packer.encode_mode12(np.zeros((64, 96), np.uint16), "x")
    with pytest.raises(ValueError):
        packer.encode_mode12(np.zeros((32, 128), np.uint16), "x")


@pytest.mark.parametrize("i", range(len(sc.PACK_CASES)))
def test_blob_assembler_rebuilds_mode12_blobs(i):
    """assemble_qr_blob (the reference's shared blob layout) around a mode-12 blob's own tiles,
    offsets and sign bits gives the blob back byte for byte (those blobs are pinned to the
    reference packer by their sha256)."""
    bv = pack_case_blob(i)
    b = packer.assemble_qr_blob(bv.mode, bv.rows, bv.cols, bv.sign_bits, bv.tiles, bv.tile_offsets, bv.tile_rows,
                                bv.ecc_group)
    assert np.array_equal(b, bv.blob)


@pytest.mark.parametrize("mode", [13, 14])
def test_hybrid_blob_round_trip(mode):
    """A synthetic mode-13/14 matrix as a blob: the finder header, tile offsets and sign bits read
    back, every tile header carries the CRC32 of its body, the parity groups XOR to zero with
    their tiles."""
    h = packer.HadTiles(mode, 1000, 256, seed=5)
    v = packer.BlobView(h.blob)
    assert (v.mode, v.rows, v.cols, v.n_tiles) == (mode, 1000, 256, h.n_tiles)
    assert np.array_equal(v.tiles, h.tiles) and np.array_equal(v.tile_offsets, h.tile_offsets)
    assert np.array_equal(v.sign_bits, h.sign_bits)
    grp = 256 // 64 * (416 if mode == 14 else 288)
    for t in range(h.n_tiles):
        tile = h.tiles[int(h.tile_offsets[t]):int(h.tile_offsets[t + 1])]
        n_r = int(tile[4:6].view(np.uint16)[0])
        body = tile[16:16 + (n_r + 7) // 8 * grp]
        assert int(tile[:4].view(np.uint32)[0]) == zlib.crc32(body.tobytes())
    ecc = v.blob[v.ecc_base_off:]
    eoffs = v.blob[64 + (v.n_tiles + 1) * 8:64 + (v.n_tiles + 1) * 8 + (v.n_ecc + 1) * 8].view(np.uint64)
    for g in range(v.n_ecc):
        par = ecc[int(eoffs[g]):int(eoffs[g + 1])].view(np.uint64).copy()
        for t in range(g * v.ecc_group, min(v.n_tiles, (g + 1) * v.ecc_group)):
            tile = h.tiles[int(h.tile_offsets[t]):int(h.tile_offsets[t + 1])].view(np.uint64)
            par[:tile.size] ^= tile
        assert not par.any()

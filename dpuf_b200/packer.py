"""Mode-12 ("Hadamard-4bit packed") weight encoder: Python front of libdpuf_pack.so.

Produces the exact bytes of the reference packer's `encode_tensor_qr_hadamard4_packed`
(dpuf_format.py:1563) for 2-D weights whose column count is a multiple of 64.

The per-tensor column signs follow `_make_had_sign_bits` (dpuf_format.py:1424-1430):
numpy's default_rng seeded with crc32(seed_name) ^ 0x9E3779B9 draws one bit per column,
packed little-endian.  Projections that share an input share a seed name
(`_hadamard_seed_name`, pack_dpuf.py:206-216): q/k/v use "blk.{l}.qkv_in", gate/up use
"blk.{l}.mlp_in", everything else its own tensor name.
"""
from __future__ import annotations

import ctypes
import os
import struct
import zlib

import numpy as np

from . import _native

MODE_QR_HAD4_PACKED = 12
MODE_QR_HAD4_ASYM = 13
MODE_QR_HAD6 = 14
TILE_ROWS = 16
QR_FINDER = struct.Struct("<B4sBHIIIIQQQ16x")  # the 64-byte finder header (dpuf_format.py:936-938)
ECC_GROUP = 64
FINDER_BYTES = 64


def _lib():
    lib = _native.load_pack()
    if not getattr(lib, "_dpuf_typed", False):
        lib.dpuf_pack_mode12_size.restype = ctypes.c_int64
        lib.dpuf_pack_mode12_size.argtypes = [ctypes.c_int32] * 4
        lib.dpuf_pack_mode12.restype = ctypes.c_int32
        lib.dpuf_pack_mode12.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32]
        lib.dpuf_gen_normal_bf16.restype = None
        lib.dpuf_gen_normal_bf16.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float,
                                             ctypes.c_void_p, ctypes.c_int32]
        lib.dpuf_pack_crc32.restype = ctypes.c_uint32
        lib.dpuf_pack_crc32.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
        lib._dpuf_typed = True
    return lib


def default_threads() -> int:
    return max(1, min(64, os.cpu_count() or 1))


def hadamard_seed_name(tensor_name: str) -> str:
    """Seed name shared by co-input projections (pack_dpuf.py:206-216)."""
    if tensor_name.startswith("blk."):
        parts = tensor_name.split(".", 2)
        if len(parts) == 3:
            l_idx, suffix = parts[1], parts[2]
            if suffix in ("attn_q.weight", "attn_k.weight", "attn_v.weight"):
                return f"blk.{l_idx}.qkv_in"
            if suffix in ("ffn_gate.weight", "ffn_up.weight"):
                return f"blk.{l_idx}.mlp_in"
    return tensor_name


def sign_bits_for(cols: int, seed_name: str) -> np.ndarray:
    """Column sign bits, cols/8 bytes (dpuf_format.py:1424-1430)."""
    seed = zlib.crc32(seed_name.encode("utf-8")) ^ 0x9E3779B9
    rng = np.random.default_rng(seed)
    flags = rng.integers(0, 2, size=cols, dtype=np.uint8)
    return np.packbits(flags, bitorder="little")


def fp32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (dpuf_format.py:74-79)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) >> 16).astype(np.uint16)


def encode_mode12(w_bf16: np.ndarray, seed_name: str, n_threads: int | None = None) -> np.ndarray:
    """Encodes a [rows, cols] bf16 (uint16 bits) matrix; returns the blob as a uint8 array."""
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    if w.ndim != 2 or w.shape[1] % 64 != 0 or min(w.shape) < 64:
        raise ValueError(f"mode 12 needs a 2-D matrix with cols % 64 == 0, got {w.shape}")
    rows, cols = w.shape
    lib = _lib()
    size = lib.dpuf_pack_mode12_size(rows, cols, TILE_ROWS, ECC_GROUP)
    if size <= 0:
        raise ValueError("bad shape for mode 12")
    out = np.empty(size, dtype=np.uint8)
    sb = sign_bits_for(cols, seed_name)
    rc = lib.dpuf_pack_mode12(w.ctypes.data, rows, cols, sb.ctypes.data, TILE_ROWS, ECC_GROUP,
                              out.ctypes.data, n_threads or default_threads())
    if rc != 0:
        raise RuntimeError(f"dpuf_pack_mode12 failed ({rc})")
    return out


def gen_normal_bf16(seed: int, stream: int, shape, sigma: float = 0.02, n_threads: int | None = None) -> np.ndarray:
    """Seeded N(0, sigma) weights rounded to bf16 (counter-based; independent of threads)."""
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.uint16)
    _lib().dpuf_gen_normal_bf16(seed & (2**64 - 1), stream & (2**64 - 1), n, sigma, out.ctypes.data,
                                n_threads or default_threads())
    return out.reshape(shape)


def assemble_qr_blob(mode: int, rows: int, cols: int, sign_bits: np.ndarray, tiles: np.ndarray,
                     tile_offsets: np.ndarray, tile_rows: int = TILE_ROWS, ecc_group: int = 64) -> np.ndarray:
    """A QR-tiled tensor blob around tiles that are already encoded, laid out as the reference's
    assembler does for every tiled mode (_assemble_qr_blob, dpuf_format.py:1182-1251): the
    64-byte finder header, the n_tiles + 1 tile offsets, the n_ecc + 1 parity offsets, the sign
    bits at the next 64-byte boundary, the tiles at the next one, then per group of `ecc_group`
    tiles their XOR as 64-bit words (each tile zero-extended to the group's longest).
    `tile_offsets` has n_tiles + 1 entries, relative to `tiles`."""
    offs = np.asarray(tile_offsets, dtype=np.uint64)
    n_tiles = offs.size - 1
    t = np.ascontiguousarray(tiles, dtype=np.uint8)
    n_ecc = (n_tiles + ecc_group - 1) // ecc_group if ecc_group > 0 else 0
    ecc_offs = np.zeros(n_ecc + 1, np.uint64)
    parity, cur = [], 0
    for g in range(n_ecc):
        ecc_offs[g] = cur
        lo, hi = g * ecc_group, min(n_tiles, (g + 1) * ecc_group)
        lens = [int(offs[i + 1] - offs[i]) for i in range(lo, hi)]
        acc = np.zeros(max(lens) // 8, np.uint64)
        for i, n in zip(range(lo, hi), lens):
            acc[:n // 8] ^= t[int(offs[i]):int(offs[i]) + n // 8 * 8].view(np.uint64)
        parity.append(acc.view(np.uint8))
        cur += acc.nbytes
    ecc_offs[n_ecc] = cur
    after_tables = QR_FINDER.size + offs.nbytes + ecc_offs.nbytes
    aux_off = after_tables + (-after_tables) % 64
    tiles_base = aux_off + sign_bits.size + (-(aux_off + sign_bits.size)) % 64
    ecc_base = tiles_base + int(offs[-1])
    hdr = QR_FINDER.pack(mode, b"QRDP", tile_rows, ecc_group, rows, cols, n_tiles, n_ecc, aux_off, tiles_base,
                         ecc_base)
    out = np.zeros(ecc_base + cur, np.uint8)
    out[:QR_FINDER.size] = np.frombuffer(hdr, np.uint8)
    out[QR_FINDER.size:QR_FINDER.size + offs.nbytes] = offs.view(np.uint8)
    out[QR_FINDER.size + offs.nbytes:after_tables] = ecc_offs.view(np.uint8)
    out[aux_off:aux_off + sign_bits.size] = sign_bits
    out[tiles_base:ecc_base] = t[:int(offs[-1])]
    pos = ecc_base
    for p in parity:
        out[pos:pos + p.size] = p
        pos += p.size
    return out


def synth_had_tiles(rows: int, cols: int, mode: int, seed: int, scale: float = 0.01):
    """A mode-13/14 tile set in the reference's layout (dpuf_avx2.c:2785-2830: a 16-byte header
    with the CRC32 of the tile body and the row count, as dpuf_format.py:1704-1709 writes it,
    then per 8-row group n64 x [8 fp16 d | 8 fp16 m], the nibbles and, for mode 14, the high bit
    pairs; tiles padded to 64 bytes) with random codes and small finite scales
    (d, m ~ N(0, scale)).  Returns (tiles, tile_offsets, sign_bits)."""
    rng = np.random.default_rng(seed)
    n64 = cols // 64
    grp = n64 * (416 if mode == 14 else 288)
    parts, offs, off = [], [], 0
    for t in range((rows + TILE_ROWS - 1) // TILE_ROWS):
        n_r = min(TILE_ROWS, rows - TILE_ROWS * t)
        n_g = (n_r + 7) // 8
        body = rng.integers(0, 256, n_g * grp, dtype=np.uint8)
        for g in range(n_g):
            dm = (rng.standard_normal(n64 * 16) * scale).astype(np.float16).view(np.uint8)
            body[g * grp:g * grp + n64 * 32] = dm
        hdr = np.zeros(16, np.uint8)
        hdr[0:4] = np.frombuffer(np.uint32(zlib.crc32(body.tobytes()) & 0xFFFFFFFF).tobytes(), np.uint8)
        hdr[4:6] = np.frombuffer(np.uint16(n_r).tobytes(), np.uint8)
        tile = np.concatenate([hdr, body, np.zeros((-(16 + body.size)) % 64, np.uint8)])
        offs.append(off)
        parts.append(tile)
        off += tile.size
    return (np.concatenate(parts), np.array(offs, np.uint64),
            rng.integers(0, 256, cols // 8, dtype=np.uint8))


class HadTiles:
    """A mode-13 (QR_HAD4_ASYM) or mode-14 (QR_HAD6) matrix with synthetic codes
    (synth_had_tiles), exposing the fields an engine descriptor takes, as BlobView does, and
    `blob`, the tensor blob a container holds (assemble_qr_blob)."""

    def __init__(self, mode: int, rows: int, cols: int, seed: int, scale: float = 0.002):
        if mode not in (13, 14) or cols % 64:
            raise ValueError("modes 13 / 14 with cols % 64 == 0")
        self.mode, self.rows, self.cols = mode, rows, cols
        self.tiles, offs, self.sign_bits = synth_had_tiles(rows, cols, mode, seed, scale)
        self.n_tiles = offs.size
        self.tile_offsets = np.append(offs, np.uint64(self.tiles.size)).astype(np.uint64)
        self.blob = assemble_qr_blob(mode, rows, cols, self.sign_bits, self.tiles, self.tile_offsets)


class BlobView:
    """Parsed view of a mode-12 blob: finder header fields and the arrays the engine binds
    (the same fields `bind_qr_weight` fills, dpuf-cli.c:1646-1756)."""

    def __init__(self, blob: np.ndarray):
        b = np.ascontiguousarray(blob, dtype=np.uint8)
        if bytes(b[1:5]) != b"QRDP":
            raise ValueError("not a QR-tiled blob (finder magic mismatch)")
        self.blob = b
        hdr = b[:64]
        self.mode = int(hdr[0])
        self.tile_rows = int(hdr[5])
        self.ecc_group = int(hdr[6:8].view(np.uint16)[0])
        self.rows, self.cols, self.n_tiles, self.n_ecc = (int(v) for v in hdr[8:24].view(np.uint32))
        self.aux_off, self.tiles_base_off, self.ecc_base_off = (int(v) for v in hdr[24:48].view(np.uint64))
        self.tile_offsets = b[64:64 + (self.n_tiles + 1) * 8].view(np.uint64)
        self.tiles = b[self.tiles_base_off:self.ecc_base_off]
        self.sign_bits = b[self.aux_off:self.aux_off + self.cols // 8]

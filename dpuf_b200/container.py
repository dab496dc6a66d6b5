"""The `.dpuf` container (magic DPUF0001): writer and zero-copy reader.

Layout (reference SPECIFICATION.md:9-53; writer save_dpuf_container, dpuf_format.py:2362-2432;
readers open_dpuf_qr_mmap, dpuf_format.py:2290-2356, and dpuf_cli_open, dpuf-cli.c:1779-1981):

    0   8 B   magic "DPUF0001"
    8   u32   number of tensors
    12  u32   CRC32 of the JSON header bytes
    16  u32   CRC32 of the payload (everything after the header)
    20  u32   JSON header length
    24  JSON  {"__metadata__": {..., "model_config": {...}, "tokenizer": {...}},
               "__tensors__": {name: [payload offset, length]}}, padded with spaces so that the
              payload starts on a 64-byte boundary of the file
    ..  payload: every tensor blob at a 64-byte aligned offset (zero padding in between)

Tensor blobs are the reference encoders' bytes: mode 12 (QR finder header, tile offsets, ECC
table, sign bits, tiles; `packer.encode_mode12`) for the matrices, or modes 13 / 14 for a
hybrid model (synthetic codes in the same blob layout, `packer.assemble_qr_blob`), mode 0 ("raw tiny":
`<BBII` mode, ndim, d0, d1, then bf16 values) for the norm gains.  The JSON keys of
`model_config` are the ones dpuf-cli.c:1191-1249 and DPUFCTransformerEngine
(dpuf_format.py:2150-2200) read.

`DpufFile` maps a file and exposes the same descriptors as `model.SyntheticModel`
(`create_args()`), pointing straight into the mapping, so any engine with the reference C ABI
can be created over it.  This module loads no native library: a process that only reads a
container (the CPU reference arm of bench.py) maps no library of this package.

    python -m dpuf_b200.container write PATH --shape qwen3-8b --seed 0 [--hybrid]
"""
from __future__ import annotations

import argparse
import json
import mmap
import os
import pathlib
import struct
import zlib

import numpy as np

from . import model as mdl
from . import packer

MAGIC = b"DPUF0001"
MODE_RAW_TINY = 0
MODE_QR_HAD4_PACKED = 12
MODES_QR_HAD_ASYM = (13, 14)  # QR_HAD4_ASYM, QR_HAD6 (the reference packer's "had4p-hybrid")


def _pad64(n: int) -> int:
    return (-n) % 64


def raw_tiny_blob(values: np.ndarray) -> bytes:
    """A 1-D fp32 vector of bf16-exact values as a mode-0 blob (dpuf_format.py:137-147)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    bits = v.view(np.uint32)
    if np.any(bits & 0xFFFF):
        raise ValueError("norm gains must be exact in bf16")
    return struct.pack("<BBII", MODE_RAW_TINY, 1, v.size, 1) + (bits >> 16).astype(np.uint16).tobytes()


def model_config_json(shape: mdl.ModelShape, has_qk_norm: bool = True) -> dict:
    return {"hidden_size": shape.hidden, "intermediate_size": shape.inter, "num_layers": shape.layers,
            "num_q_heads": shape.n_q, "num_kv_heads": shape.n_kv, "head_dim": shape.head_dim,
            "vocab_size": shape.vocab, "max_seq_len": shape.max_seq, "has_qk_norm": bool(has_qk_norm),
            "rms_eps": shape.rms_eps, "rope_theta": shape.rope_theta, "tie_word_embeddings": bool(shape.tied),
            "model_type": "qwen3"}


def byte_symbols() -> list[str]:
    """The byte-level BPE alphabet (GPT-2's byte-to-unicode map, which the reference CLI's
    tokenizer inverts, dpuf-cli.c:553-568): printable bytes stand for themselves, the others for
    code points 256 + n in byte order."""
    keep = set(range(33, 127)) | set(range(161, 173)) | set(range(174, 256))
    out, n = [], 0
    for b in range(256):
        if b in keep:
            out.append(chr(b))
        else:
            out.append(chr(256 + n))
            n += 1
    return out


def synthetic_tokenizer(vocab: int) -> dict:
    """A tokenizer object for the container's metadata (the keys dpuf-cli.c:1309-1400 reads) for
    random-init models: ids 0..255 are the 256 byte symbols, so any text encodes byte by byte (no
    merges), and every other id decodes to "[id]".  No end-of-sequence id, raw chat format."""
    syms = byte_symbols()
    return {"vocab": syms + [f"[{i}]" for i in range(256, vocab)], "merges": [], "eos_token_ids": [],
            "bos_token_id": None, "add_bos": False, "chat_format": "raw"}


def tensor_order(shape: mdl.ModelShape) -> list[str]:
    names = ["token_embd.weight"]
    if not shape.tied:
        names.append("output.weight")
    names.append("output_norm.weight")
    for l in range(shape.layers):
        names += [f"blk.{l}.{s}" for s, _, _ in shape.linear_shapes()]
        names += [f"blk.{l}.attn_norm.weight", f"blk.{l}.ffn_norm.weight", f"blk.{l}.attn_q_norm.weight",
                  f"blk.{l}.attn_k_norm.weight"]
    return names


def write(path: str | os.PathLike, m: mdl.ModelData, tokenizer: dict | None = None,
          extra_meta: dict | None = None) -> int:
    """Writes model `m` (mode-12 blobs and norm gains) as a DPUF0001 container; returns the
    file size.  The file is written under a temporary name and renamed when complete."""
    path = pathlib.Path(path)
    names = [n for n in tensor_order(m.shape) if n in m.blobs or n in m.norms]
    blobs: list[bytes | np.ndarray] = []
    index, offset, pay_crc = {}, 0, 0
    pads = []
    for n in names:
        b = m.blobs[n].blob if n in m.blobs else np.frombuffer(raw_tiny_blob(m.norms[n]), np.uint8)
        pad = _pad64(offset)
        if pad:
            pay_crc = zlib.crc32(b"\x00" * pad, pay_crc)
            offset += pad
        pads.append(pad)
        index[n] = [offset, int(b.size)]
        pay_crc = zlib.crc32(memoryview(b), pay_crc)
        offset += int(b.size)
        blobs.append(b)
    hybrid = any(getattr(b, "mode", MODE_QR_HAD4_PACKED) != MODE_QR_HAD4_PACKED for b in m.blobs.values())
    meta = {"format": "DPUF / LR-FLAC", "min_reader_version": "1.2.0", "model_name": m.shape.name,
            "architecture": "qwen3",
            "compression_mode": "had4p-hybrid (modes 13/14)" if hybrid else "had4p (mode 12)",
            "num_tensors": len(names),
            "payload_bytes": offset, "model_config": model_config_json(m.shape, m.has_qk_norm)}
    if tokenizer is not None:
        meta["tokenizer"] = tokenizer
    if extra_meta:
        meta.update(extra_meta)
    hdr = json.dumps({"__metadata__": meta, "__tensors__": index}, separators=(",", ":"),
                     ensure_ascii=False).encode("utf-8")
    hdr += b" " * _pad64(24 + len(hdr))
    top = struct.pack("<8sIIII", MAGIC, len(names), zlib.crc32(hdr) & 0xFFFFFFFF, pay_crc & 0xFFFFFFFF, len(hdr))
    tmp = path.with_name(path.name + ".part")
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(tmp, "wb") as f:
        f.write(top)
        f.write(hdr)
        for b, pad in zip(blobs, pads):
            if pad:
                f.write(b"\x00" * pad)
            f.write(memoryview(b))
    os.replace(tmp, path)
    return 24 + len(hdr) + offset


class DpufFile(mdl.ModelData):
    """A DPUF0001 container mapped read-only; blobs and norm gains are views into the mapping
    (norm gains are widened from bf16 to fp32 copies, as the reference loaders do)."""

    def __init__(self, path: str | os.PathLike, verify_payload: bool = False, max_seq_len: int | None = None):
        self.path = pathlib.Path(path)
        self._f = open(self.path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        mm = self._mm
        if len(mm) < 24:
            raise ValueError("file too short for a DPUF header")
        magic, n_tensors, hdr_crc, pay_crc, hdr_len = struct.unpack("<8sIIII", mm[:24])
        if magic != MAGIC:
            raise ValueError(f"not a DPUF0001 container (magic {magic!r})")
        hdr = bytes(mm[24:24 + hdr_len])
        if zlib.crc32(hdr) & 0xFFFFFFFF != hdr_crc:
            raise ValueError("header CRC32 mismatch")
        base = 24 + hdr_len
        if verify_payload and zlib.crc32(memoryview(mm)[base:]) & 0xFFFFFFFF != pay_crc:
            raise ValueError("payload CRC32 mismatch")
        obj = json.loads(hdr.decode("utf-8"))
        self.meta = obj.get("__metadata__", {})
        index = obj["__tensors__"]
        if len(index) != n_tensors:
            raise ValueError("tensor count does not match the header")
        u8 = np.frombuffer(mm, dtype=np.uint8)
        self.blobs, self.norms = {}, {}
        for name, (off, length) in index.items():
            view = u8[base + int(off): base + int(off) + int(length)]
            mode = int(view[0])
            if mode == MODE_QR_HAD4_PACKED or mode in MODES_QR_HAD_ASYM:
                self.blobs[name] = packer.BlobView(view)
            elif mode == MODE_RAW_TINY:
                _, ndim, d0, d1 = struct.unpack("<BBII", bytes(view[:10]))
                raw = view[10:]
                if d1 == 2 and raw.size == d0 * 4:
                    self.norms[name] = raw.view(np.float32).copy()
                else:
                    self.norms[name] = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).copy()
            else:
                raise ValueError(f"{name}: mode {mode} is not supported by this engine")
        cfg = self.meta.get("model_config", {})
        tok = self.blobs["token_embd.weight"]
        self.has_qk_norm = "blk.0.attn_q_norm.weight" in self.norms
        n_layers = 0
        while f"blk.{n_layers}.attn_q.weight" in self.blobs:
            n_layers += 1
        hd = int(cfg.get("head_dim", 128))
        self.shape = mdl.ModelShape(
            name=str(self.meta.get("model_name", self.path.stem)), hidden=int(cfg.get("hidden_size", tok.cols)),
            inter=int(cfg.get("intermediate_size", self.blobs["blk.0.ffn_gate.weight"].rows)), layers=n_layers,
            n_q=int(cfg.get("num_q_heads", self.blobs["blk.0.attn_q.weight"].rows // hd)),
            n_kv=int(cfg.get("num_kv_heads", self.blobs["blk.0.attn_k.weight"].rows // hd)), head_dim=hd,
            vocab=int(cfg.get("vocab_size", tok.rows)), tied="output.weight" not in self.blobs,
            max_seq=int(max_seq_len or cfg.get("max_seq_len", 2048)),
            rope_theta=float(cfg.get("rope_theta", 1e6)), rms_eps=float(cfg.get("rms_eps", 1e-6)))
        self._build_descs()

    def close(self) -> None:
        self.blobs, self.norms = {}, {}
        if getattr(self, "_mm", None) is not None:
            try:
                self._mm.close()
            except BufferError:
                pass  # views still alive; the mapping goes with them
            self._mm = None
            self._f.close()


def write_synthetic(path: str | os.PathLike, shape_name: str, seed: int = 0, hybrid: bool = False) -> int:
    """Builds the random-init model `shape_name` (model.SHAPES) and writes it as a container;
    `hybrid`: every matrix in mode 13 or 14 as the reference's had4p-hybrid packing assigns them
    (model.hybrid_mode), with synthetic codes."""
    m = mdl.SyntheticModel(mdl.SHAPES[shape_name], seed=seed, hybrid=hybrid)
    return write(path, m, tokenizer=synthetic_tokenizer(m.shape.vocab), extra_meta={"synthetic_seed": seed})


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="write a random-init model as a DPUF0001 container")
    sub = ap.add_subparsers(dest="cmd", required=True)
    w = sub.add_parser("write")
    w.add_argument("path")
    w.add_argument("--shape", default="qwen3-8b", choices=sorted(mdl.SHAPES))
    w.add_argument("--seed", type=int, default=0)
    w.add_argument("--hybrid", action="store_true", help="modes 13/14 as the had4p-hybrid packing assigns them")
    args = ap.parse_args(argv)
    if args.cmd == "write":
        n = write_synthetic(args.path, args.shape, args.seed, args.hybrid)
        print(json.dumps({"path": args.path, "bytes": n}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

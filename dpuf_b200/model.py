"""Model description, random-init synthetic models, and the ctypes mirrors of the C ABI structs.

The structs mirror include/dpuf_kernels.h byte for byte (the reference's ctypes mirrors are
dpuf_format.py:2060-2114).  `SyntheticModel` builds a random-init decoder in mode-12 layout
in host memory: weights w = 0.02 * N(0,1) (seeded, rounded to bf16 as the reference packer
does, pack_dpuf.py:105-108), quantised by the mode-12 encoder, norm gains 1.0 unless
`norm_jitter` asks for random gains (used by tests to exercise the norm-gain indexing).
"""
from __future__ import annotations

import ctypes
import dataclasses
import zlib

import numpy as np

from . import packer


class DpufWeightDesc(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("rows", ctypes.c_int32),
        ("cols", ctypes.c_int32),
        ("n_tiles", ctypes.c_int32),
        ("tensor_base", ctypes.c_void_p),
        ("tile_offsets", ctypes.c_void_p),
        ("col_scale", ctypes.c_void_p),
        ("sign_bits", ctypes.c_void_p),
    ]


class DpufModelConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int32),
        ("intermediate_size", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32),
        ("has_qk_norm", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("n_threads", ctypes.c_int32),
        ("use_llama3_rope", ctypes.c_int32),
        ("rope_factor", ctypes.c_float),
        ("rope_low_freq", ctypes.c_float),
        ("rope_high_freq", ctypes.c_float),
        ("rope_orig_max_pos", ctypes.c_int32),
        ("kv_type", ctypes.c_int32),
        ("has_mrope", ctypes.c_int32),
        ("mrope_section", ctypes.c_int32 * 3),
        ("mrope_interleaved", ctypes.c_int32),
    ]


class DpufLayerWeights(ctypes.Structure):
    _fields_ = [
        ("attn_norm", ctypes.c_void_p),
        ("attn_q_norm", ctypes.c_void_p),
        ("attn_k_norm", ctypes.c_void_p),
        ("ffn_norm", ctypes.c_void_p),
        ("w_q", DpufWeightDesc),
        ("w_k", DpufWeightDesc),
        ("w_v", DpufWeightDesc),
        ("w_o", DpufWeightDesc),
        ("w_gate", DpufWeightDesc),
        ("w_up", DpufWeightDesc),
        ("w_down", DpufWeightDesc),
    ]


assert ctypes.sizeof(DpufWeightDesc) == 48
assert ctypes.sizeof(DpufModelConfig) == 92
assert ctypes.sizeof(DpufLayerWeights) == 368


@dataclasses.dataclass(frozen=True)
class ModelShape:
    name: str
    hidden: int
    inter: int
    layers: int
    n_q: int
    n_kv: int
    head_dim: int
    vocab: int
    tied: bool
    max_seq: int = 2304
    rope_theta: float = 1e6
    rms_eps: float = 1e-6

    @property
    def q_dim(self) -> int:
        return self.n_q * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv * self.head_dim

    def linear_shapes(self):
        """(tensor name suffix, rows, cols) of one layer's projections (GGUF names)."""
        H, I = self.hidden, self.inter
        return [("attn_q.weight", self.q_dim, H), ("attn_k.weight", self.kv_dim, H),
                ("attn_v.weight", self.kv_dim, H), ("attn_output.weight", H, self.q_dim),
                ("ffn_gate.weight", I, H), ("ffn_up.weight", I, H), ("ffn_down.weight", H, I)]

    def weight_bytes_per_token(self) -> int:
        """Mode-12 bytes streamed by one decode step: every layer matrix plus the LM head
        (tile headers and padding included, i.e. the bytes the GEMVs read)."""
        def mat(rows, cols):
            n_tiles = (rows + 15) // 16
            raw = 16 + 2 * (cols // 32) * 144
            return n_tiles * (raw + (-raw) % 64)
        per_layer = sum(mat(r, c) for _, r, c in self.linear_shapes())
        return self.layers * per_layer + mat(self.vocab, self.hidden)

    def expanded_bytes_per_layer(self) -> int:
        """Bytes of one layer's expanded copies, which the tensor-core GEMM streams for M > 1:
        per 128-row group (8 tiles) and 32-column block, 4,096 B of s8 weights and 256 B of
        fp16 row scales."""
        return sum(((r + 15) // 16 + 7) // 8 * (c // 32) * 4352 for _, r, c in self.linear_shapes())


QWEN3_0_6B = ModelShape("qwen3-0.6b", 1024, 3072, 28, 16, 8, 128, 151936, tied=True)
QWEN3_8B = ModelShape("qwen3-8b", 4096, 12288, 36, 32, 8, 128, 151936, tied=False)
TINY = ModelShape("tiny", 256, 512, 2, 4, 2, 64, 4096, tied=False, max_seq=512)
TINY_ZONE = ModelShape("tiny-zone", 256, 512, 2, 4, 2, 64, 40960, tied=True, max_seq=512)
TINY_MHA = ModelShape("tiny-mha", 256, 512, 2, 3, 3, 64, 4096, tied=False, max_seq=512)
# the 8B shape's FFN width on two small layers (the persistent kernel's distributed down-input prep)
TINY_WIDE = ModelShape("tiny-wide", 1024, 12288, 2, 8, 4, 128, 4096, tied=False, max_seq=512)
# three query heads per KV head: one pair and one lone head in every group
TINY_G3 = ModelShape("tiny-g3", 256, 512, 2, 6, 2, 64, 4096, tied=False, max_seq=512)
# a small model with the configurations' longest context (fp32 KV cache beyond 2048 positions)
TINY_LONG = ModelShape("tiny-long", 256, 512, 2, 4, 2, 64, 4096, tied=False, max_seq=2304)
# the 8B shape cut to four layers (same per-layer work and LM head): profiler captures of the
# decode kernel that fit a few GB on the device
QWEN3_8B_L4 = dataclasses.replace(QWEN3_8B, name="qwen3-8b-l4", layers=4)
SHAPES = {s.name: s for s in (QWEN3_0_6B, QWEN3_8B, QWEN3_8B_L4, TINY, TINY_ZONE, TINY_MHA, TINY_WIDE, TINY_G3,
                              TINY_LONG)}


def _stream_id(name: str) -> int:
    return zlib.crc32(name.encode("utf-8"))


class ModelData:
    """A mode-12 model in host memory: `blobs` (tensor name -> packer.BlobView), `norms` (name ->
    fp32 gains) and `shape`, with the C-ABI descriptors built over them (`create_args`).  The
    arrays must stay alive while an engine created from them is (the reference engine borrows
    them; this library's engine copies them at create)."""

    shape: ModelShape
    blobs: dict
    norms: dict
    has_qk_norm: bool = True

    def desc(self, name: str) -> DpufWeightDesc:
        bv = self.blobs[name]
        d = DpufWeightDesc()
        d.mode = bv.mode
        d.rows = bv.rows
        d.cols = bv.cols
        d.n_tiles = bv.n_tiles
        d.tensor_base = bv.tiles.ctypes.data
        d.tile_offsets = bv.tile_offsets.ctypes.data
        d.col_scale = None
        d.sign_bits = bv.sign_bits.ctypes.data
        return d

    def _build_descs(self) -> None:
        s = self.shape
        cfg = DpufModelConfig()
        cfg.hidden_size = s.hidden
        cfg.intermediate_size = s.inter
        cfg.num_layers = s.layers
        cfg.num_q_heads = s.n_q
        cfg.num_kv_heads = s.n_kv
        cfg.head_dim = s.head_dim
        cfg.vocab_size = s.vocab
        cfg.max_seq_len = s.max_seq
        cfg.has_qk_norm = 1 if self.has_qk_norm else 0
        cfg.rms_eps = s.rms_eps
        cfg.rope_theta = s.rope_theta
        cfg.n_threads = 8
        cfg.kv_type = 0
        self.cfg = cfg
        arr = (DpufLayerWeights * s.layers)()
        keys = ["w_q", "w_k", "w_v", "w_o", "w_gate", "w_up", "w_down"]
        for l in range(s.layers):
            lw = arr[l]
            lw.attn_norm = self.norms[f"blk.{l}.attn_norm.weight"].ctypes.data
            if self.has_qk_norm:
                lw.attn_q_norm = self.norms[f"blk.{l}.attn_q_norm.weight"].ctypes.data
                lw.attn_k_norm = self.norms[f"blk.{l}.attn_k_norm.weight"].ctypes.data
            lw.ffn_norm = self.norms[f"blk.{l}.ffn_norm.weight"].ctypes.data
            for key, (suffix, _, _) in zip(keys, s.linear_shapes()):
                setattr(lw, key, self.desc(f"blk.{l}.{suffix}"))
        self.layers = arr
        self.tok = self.desc("token_embd.weight")
        self.lm = self.desc("output.weight" if "output.weight" in self.blobs else "token_embd.weight")
        self.out_norm = self.norms["output_norm.weight"]

    def create_args(self):
        """Arguments of dpuf_engine_create (reference dpuf_kernels.h:316-322)."""
        return (ctypes.byref(self.cfg), self.layers, ctypes.byref(self.tok), ctypes.byref(self.lm),
                self.out_norm.ctypes.data)


def hybrid_mode(name: str) -> int:
    """The mode the reference packer's "had4p-hybrid" setting gives a matrix (pack_dpuf.py:249-266):
    14 (QR_HAD6) for the down projection, k and v, the o projection of even layers and the
    untied LM head; 13 (QR_HAD4_ASYM) for the rest."""
    l_idx = int(name.split(".")[1]) if name.startswith("blk.") else -1
    if (name.endswith(".ffn_down.weight") or name.endswith(".attn_v.weight") or name.endswith(".attn_k.weight")
            or (name.endswith(".attn_output.weight") and l_idx >= 0 and l_idx % 2 == 0) or name == "output.weight"):
        return 14
    return 13


class SyntheticModel(ModelData):
    """Random-init model held in host memory, with C-ABI descriptors: mode-12 matrices encoded by
    the packer, or (hybrid) every matrix in mode 13 or 14 as the reference's had4p-hybrid setting
    assigns them, with synthetic codes (packer.HadTiles)."""

    def __init__(self, shape: ModelShape, seed: int = 0, norm_jitter: float = 0.0, n_threads: int | None = None,
                 hybrid: bool = False):
        self.shape = shape
        self.seed = seed
        self.blobs: dict[str, packer.BlobView] = {}
        self.norms: dict[str, np.ndarray] = {}
        s = shape
        rng = np.random.default_rng(seed + 7919)

        def norm(name: str, n: int) -> np.ndarray:
            g = np.ones(n, dtype=np.float32)
            if norm_jitter > 0:
                g = (g + rng.standard_normal(n).astype(np.float32) * np.float32(norm_jitter))
                g = packer.fp32_to_bf16(g).astype(np.uint32) << 16
                g = g.view(np.float32)
            self.norms[name] = np.ascontiguousarray(g, dtype=np.float32)
            return self.norms[name]

        def mat(name: str, rows: int, cols: int):
            if hybrid:
                self.blobs[name] = packer.HadTiles(hybrid_mode(name), rows, cols, seed * 1000003 + _stream_id(name))
                return
            w = packer.gen_normal_bf16(seed, _stream_id(name), (rows, cols), 0.02, n_threads)
            self.blobs[name] = packer.BlobView(packer.encode_mode12(w, packer.hadamard_seed_name(name), n_threads))

        mat("token_embd.weight", s.vocab, s.hidden)
        if not s.tied:
            mat("output.weight", s.vocab, s.hidden)
        norm("output_norm.weight", s.hidden)
        for l in range(s.layers):
            for suffix, rows, cols in s.linear_shapes():
                mat(f"blk.{l}.{suffix}", rows, cols)
            norm(f"blk.{l}.attn_norm.weight", s.hidden)
            norm(f"blk.{l}.ffn_norm.weight", s.hidden)
            norm(f"blk.{l}.attn_q_norm.weight", s.head_dim)
            norm(f"blk.{l}.attn_k_norm.weight", s.head_dim)
        self._build_descs()


def prompt_ids(n: int, vocab: int, seed: int = 0) -> np.ndarray:
    """Prompt of n ids uniform in [0, vocab) from numpy's default_rng(seed)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)

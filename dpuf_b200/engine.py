"""Python front of the CUDA engine, mirroring the reference's ctypes driver
`dpuf_format.DPUFCTransformerEngine` (dpuf_format.py:2130-2287): same method names, argument
meaning and RuntimeError on a nonzero return code.  All work happens in libdpuf_cuda.so; this
module only marshals arguments.  There is no fallback: a missing library or GPU is an error.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native

_I32 = ctypes.c_int32
_VP = ctypes.c_void_p


def cuda_lib() -> ctypes.CDLL:
    lib = _native.load_cuda()
    if getattr(lib, "_dpuf_typed", False):
        return lib
    lib.dpuf_engine_create.restype = _VP
    lib.dpuf_engine_create.argtypes = [_VP] * 5
    lib.dpuf_engine_destroy.argtypes = [_VP]
    lib.dpuf_engine_reset_cache.argtypes = [_VP]
    lib.dpuf_engine_set_slot.restype = _I32
    lib.dpuf_engine_set_slot.argtypes = [_VP, _I32]
    lib.dpuf_engine_get_slot.restype = _I32
    lib.dpuf_engine_get_slot.argtypes = [_VP]
    lib.dpuf_engine_reset_slot.argtypes = [_VP, _I32]
    lib.dpuf_engine_slot_memory.restype = ctypes.c_size_t
    lib.dpuf_engine_slot_memory.argtypes = [_VP]
    lib.dpuf_engine_num_slots.restype = _I32
    lib.dpuf_engine_num_slots.argtypes = [_VP]
    lib.dpuf_engine_freeze_prefix.restype = _I32
    lib.dpuf_engine_freeze_prefix.argtypes = [_VP, _I32, _I32]
    lib.dpuf_engine_apply_prefix.restype = _I32
    lib.dpuf_engine_apply_prefix.argtypes = [_VP, _I32, _I32]
    lib.dpuf_engine_get_prefix_len.restype = _I32
    lib.dpuf_engine_get_prefix_len.argtypes = [_VP, _I32]
    lib.dpuf_engine_forward_batch.restype = _I32
    lib.dpuf_engine_forward_batch.argtypes = [_VP, _I32, _VP, _I32, _I32, _VP]
    lib.dpuf_engine_forward_batch_ex.restype = _I32
    lib.dpuf_engine_forward_batch_ex.argtypes = [_VP, _I32, _VP, _I32, _VP, _VP, _VP, _VP, _VP, _I32, _VP]
    lib.dpuf_engine_forward_token.restype = _I32
    lib.dpuf_engine_forward_token.argtypes = [_VP, _I32, _I32, _VP]
    lib.dpuf_cuda_forward_greedy.restype = _I32
    lib.dpuf_cuda_forward_greedy.argtypes = [_VP, _I32, _VP, _I32, _VP]
    lib.dpuf_cuda_read_logits.restype = _I32
    lib.dpuf_cuda_read_logits.argtypes = [_VP, _I32, _VP]
    lib.dpuf_cuda_set_option.restype = _I32
    lib.dpuf_cuda_set_option.argtypes = [_VP, ctypes.c_char_p, ctypes.c_int64]
    lib.dpuf_cuda_zone_head.restype = _I32
    lib.dpuf_cuda_zone_head.argtypes = [_VP, _I32, _VP, _I32, ctypes.c_float, _VP, _VP, _VP]
    lib.dpuf_cuda_matmul_dev_timed.restype = _I32
    lib.dpuf_cuda_matmul_dev_timed.argtypes = [_VP, _I32, _I32, _VP, _VP, _I32, _VP, _VP]
    lib.dpuf_cuda_decode_greedy.restype = _I32
    lib.dpuf_cuda_decode_greedy.argtypes = [_VP, _I32, _I32, _I32, _VP, _VP]
    lib.dpuf_cuda_persistent_decode.restype = _I32
    lib.dpuf_cuda_persistent_decode.argtypes = [_VP, _VP]
    lib.dpuf_cuda_zone_info.restype = _I32
    lib.dpuf_cuda_zone_info.argtypes = [_VP, _VP, _VP, _VP, _VP]
    lib.dpuf_cuda_last_error.restype = ctypes.c_char_p
    lib.dpuf_cuda_w12_upload.restype = _VP
    lib.dpuf_cuda_w12_upload.argtypes = [_VP]
    lib.dpuf_cuda_w12_free.argtypes = [_VP]
    lib.dpuf_cuda_matmul_dev.restype = _I32
    lib.dpuf_cuda_matmul_dev.argtypes = [_VP, _I32, _VP, _VP, _VP]
    lib.dpuf_matmul_qr_hadamard4_packed_f32.restype = None
    lib.dpuf_matmul_qr_hadamard4_packed_f32.argtypes = [_I32] * 4 + [_VP] * 5
    lib.dpuf_embed_qr_hadamard4_packed_f32.restype = None
    lib.dpuf_embed_qr_hadamard4_packed_f32.argtypes = [_I32, _I32] + [_VP] * 5
    lib.dpuf_cuda_prepare_expf_table.restype = ctypes.c_int64
    lib.dpuf_cuda_matmul_noalloc.restype = _I32
    lib.dpuf_cuda_matmul_noalloc.argtypes = [_I32] * 4 + [_VP] * 6
    lib.dpuf_cuda_decode_batch.restype = _I32
    lib.dpuf_cuda_decode_batch.argtypes = [_VP, _I32, _VP, _VP, _VP, _VP, _VP]
    lib.dpuf_cuda_tp_handle.restype = _I32
    lib.dpuf_cuda_tp_handle.argtypes = [_VP, _I32, _I32, _VP]
    lib.dpuf_cuda_tp_attach.restype = _I32
    lib.dpuf_cuda_tp_attach.argtypes = [_VP, _VP]
    lib.dpuf_cuda_sample_seed.restype = ctypes.c_uint64
    lib.dpuf_cuda_sample_seed.argtypes = []
    lib.dpuf_cuda_sample_token.restype = _I32
    lib.dpuf_cuda_sample_token.argtypes = [_VP, _I32, ctypes.c_float, _VP]
    lib._dpuf_typed = True
    return lib


TP_BLOB_BYTES = 256  # DPUF_CUDA_TP_BLOB_BYTES


def torch_all_gather(group=None):
    """all_gather for CudaTransformerEngine.tp_attach over a torch.distributed group."""
    import torch.distributed as dist

    def gather(b: bytes) -> list[bytes]:
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, b, group=group)
        return out

    return gather


def last_error() -> str:
    return (cuda_lib().dpuf_cuda_last_error() or b"").decode()


class CudaTransformerEngine:
    """The engine over a model given as C-ABI structs (e.g. `model.SyntheticModel`)."""

    def __init__(self, model, options: dict | None = None):
        self.lib = cuda_lib()
        self.model = model
        self.vocab_size = model.shape.vocab
        self._handle = self.lib.dpuf_engine_create(*model.create_args())
        if not self._handle:
            raise RuntimeError(f"dpuf_engine_create failed: {last_error()}")
        for k, v in (options or {}).items():
            if self.lib.dpuf_cuda_set_option(self._handle, k.encode(), int(v)) != 0:
                raise ValueError(f"unknown engine option {k}")

    def set_option(self, name: str, value: int) -> None:
        """dpuf_cuda_set_option (include/dpuf_cuda.h): engine options and test hooks."""
        if self.lib.dpuf_cuda_set_option(self._handle, name.encode(), int(value)) != 0:
            raise ValueError(f"engine option {name}={value} rejected")

    # --- reference driver surface (dpuf_format.py:2250-2287)
    def reset_cache(self):
        if self._handle:
            self.lib.dpuf_engine_reset_cache(self._handle)

    reset = reset_cache

    def forward_token(self, token_id: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab_size, dtype=np.float32)
        rc = self.lib.dpuf_engine_forward_token(self._handle, int(token_id), int(pos), out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"dpuf_engine_forward_token failed with rc={rc}: {last_error()}")
        return out

    def forward_batch(self, token_ids, pos0: int = 0, only_last_logits=True) -> np.ndarray:
        ids = np.ascontiguousarray(token_ids, dtype=np.int32).ravel()
        m = int(ids.size)
        if only_last_logits == 2:
            rc = self.lib.dpuf_engine_forward_batch(self._handle, m, ids.ctypes.data, int(pos0), 2, None)
            if rc != 0:
                raise RuntimeError(f"dpuf_engine_forward_batch failed with rc={rc}: {last_error()}")
            return np.empty((0, self.vocab_size), np.float32)
        out_m = 1 if only_last_logits else m
        out = np.empty((out_m, self.vocab_size), dtype=np.float32)
        rc = self.lib.dpuf_engine_forward_batch(self._handle, m, ids.ctypes.data, int(pos0),
                                                1 if only_last_logits else 0, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"dpuf_engine_forward_batch failed with rc={rc}: {last_error()}")
        return out

    def forward(self, ids, pos0: int, only_last: int = 1):
        """Oracle-compatible spelling used by the parity tests."""
        return self.forward_batch(ids, pos0, only_last)

    def forward_greedy(self, token_ids, pos0: int) -> int:
        ids = np.ascontiguousarray(token_ids, dtype=np.int32).ravel()
        nxt = np.zeros(1, np.int32)
        rc = self.lib.dpuf_cuda_forward_greedy(self._handle, int(ids.size), ids.ctypes.data, int(pos0), nxt.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"dpuf_cuda_forward_greedy failed with rc={rc}: {last_error()}")
        return int(nxt[0])

    def decode_greedy(self, first_id: int, pos0: int, n_steps: int) -> tuple[list[int], float]:
        """n_steps greedy steps with the token fed back on the device; (ids, device ms)."""
        ids = np.zeros(n_steps, np.int32)
        ms = ctypes.c_float()
        rc = self.lib.dpuf_cuda_decode_greedy(self._handle, int(first_id), int(pos0), int(n_steps), ids.ctypes.data,
                                              ctypes.byref(ms))
        if rc != 0:
            raise RuntimeError(f"dpuf_cuda_decode_greedy failed with rc={rc}: {last_error()}")
        return [int(i) for i in ids], float(ms.value)

    def decode_batch(self, slots, ids, pos, want_logits: bool = False):
        """One greedy step of independent sequences (row i: slot slots[i], position pos[i], input
        ids[i]); returns the next ids (and the [n][vocab] logits when asked)."""
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        n = slots.size
        nxt = np.zeros(n, np.int32)
        logits = np.empty((n, self.vocab_size), np.float32) if want_logits else None
        rc = self.lib.dpuf_cuda_decode_batch(self._handle, n, slots.ctypes.data, ids.ctypes.data, pos.ctypes.data,
                                             nxt.ctypes.data, logits.ctypes.data if want_logits else None)
        if rc != 0:
            raise RuntimeError(f"dpuf_cuda_decode_batch failed with rc={rc}: {last_error()}")
        return (nxt, logits) if want_logits else nxt

    def persistent_decode(self) -> tuple[bool, str]:
        """Whether batch-1 steps run as the persistent kernel, and why not."""
        why = ctypes.c_char_p()
        on = self.lib.dpuf_cuda_persistent_decode(self._handle, ctypes.byref(why))
        return on == 1, (why.value or b"").decode()

    def tp_attach(self, rank: int, world: int, all_gather) -> None:
        """Tensor parallelism of batch-1 decode steps over `world` processes (one GPU each):
        publishes this rank's exchange buffer, all-gathers every rank's description with
        `all_gather(bytes) -> list[bytes]` (in rank order; e.g. over the caller's
        torch.distributed group) and maps the other ranks' buffers.  Every rank must then make
        the same engine calls in the same order."""
        blob = np.zeros(TP_BLOB_BYTES, np.uint8)
        rc = self.lib.dpuf_cuda_tp_handle(self._handle, int(rank), int(world), blob.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"dpuf_cuda_tp_handle failed with rc={rc}: {last_error()}")
        blobs = all_gather(blob.tobytes())
        if len(blobs) != world or any(len(b) != TP_BLOB_BYTES for b in blobs):
            raise ValueError("all_gather must return one blob per rank")
        allb = np.frombuffer(b"".join(blobs), np.uint8).copy()
        rc = self.lib.dpuf_cuda_tp_attach(self._handle, allb.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"dpuf_cuda_tp_attach failed with rc={rc}: {last_error()}")

    def zone_info(self):
        used, exited = np.zeros(1, np.int32), np.zeros(1, np.int32)
        b1, b2 = np.zeros(1, np.float32), np.zeros(1, np.float32)
        self.lib.dpuf_cuda_zone_info(self._handle, used.ctypes.data, exited.ctypes.data, b1.ctypes.data, b2.ctypes.data)
        return int(used[0]), int(exited[0]), float(b1[0]), float(b2[0])

    # --- slots and prefixes (dpuf_kernels.h:325-333)
    def set_slot(self, slot: int) -> int:
        return self.lib.dpuf_engine_set_slot(self._handle, slot)

    def get_slot(self) -> int:
        return self.lib.dpuf_engine_get_slot(self._handle)

    def reset_slot(self, slot: int) -> None:
        self.lib.dpuf_engine_reset_slot(self._handle, slot)

    def slot_memory(self) -> int:
        return self.lib.dpuf_engine_slot_memory(self._handle)

    def num_slots(self) -> int:
        return self.lib.dpuf_engine_num_slots(self._handle)

    def freeze_prefix(self, prefix_id: int, prefix_len: int) -> int:
        return self.lib.dpuf_engine_freeze_prefix(self._handle, prefix_id, prefix_len)

    def apply_prefix(self, slot: int, prefix_id: int) -> int:
        return self.lib.dpuf_engine_apply_prefix(self._handle, slot, prefix_id)

    def get_prefix_len(self, prefix_id: int) -> int:
        return self.lib.dpuf_engine_get_prefix_len(self._handle, prefix_id)

    def close(self):
        if getattr(self, "_handle", None):
            self.lib.dpuf_engine_destroy(self._handle)
            self._handle = None

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        self.close()

    def __del__(self):
        self.close()


def matmul(M: int, blob, x: np.ndarray) -> np.ndarray:
    """Standalone mode-12 matmul through the drop-in symbol (host in, host out)."""
    lib = cuda_lib()
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((M, blob.rows), dtype=np.float32)
    lib.dpuf_matmul_qr_hadamard4_packed_f32(M, blob.rows, blob.cols, blob.n_tiles, x.ctypes.data, blob.tiles.ctypes.data,
                                            blob.tile_offsets.ctypes.data, blob.sign_bits.ctypes.data, out.ctypes.data)
    err = last_error()
    if err:
        raise RuntimeError(err)
    return out


def upload(blob):
    """Device-resident copy of a mode-12 matrix (dpuf_cuda_w12_upload); free with w12_free."""
    from . import model as mdl

    lib = cuda_lib()
    d = mdl.DpufWeightDesc(12, blob.rows, blob.cols, blob.n_tiles, blob.tiles.ctypes.data,
                           blob.tile_offsets.ctypes.data, None, blob.sign_bits.ctypes.data)
    h = lib.dpuf_cuda_w12_upload(ctypes.byref(d))
    if not h:
        raise RuntimeError(f"dpuf_cuda_w12_upload failed: {last_error()}")
    return h


def w12_free(h) -> None:
    cuda_lib().dpuf_cuda_w12_free(h)


def zone_head(blob, x: np.ndarray, zone_tiles: int, margin: float):
    """LM head with the Zone-A early exit on hidden vectors x[n][cols] (already normalised):
    (ids, exits, device ms) from dpuf_cuda_zone_head."""
    import torch

    lib = cuda_lib()
    h = upload(blob)
    try:
        xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
        n = x.shape[0]
        ids = np.zeros(n, np.int32)
        exits = np.zeros(n, np.int32)
        ms = ctypes.c_float()
        rc = lib.dpuf_cuda_zone_head(h, n, ctypes.c_void_p(xd.data_ptr()), int(zone_tiles), float(margin),
                                     ids.ctypes.data, exits.ctypes.data, ctypes.byref(ms))
        if rc != 0:
            raise RuntimeError(f"dpuf_cuda_zone_head failed with rc={rc}: {last_error()}")
        return ids, exits, float(ms.value)
    finally:
        w12_free(h)


class Sampler:
    """Token sampler of the engine's callers: the reference CLI's sample_token
    (dpuf-cli.c:1997-2027) with its xorshift64* generator (dpuf-cli.c:1987-1995), whose state
    this object carries (the reference keeps one process-global state, starting at
    dpuf_cuda_sample_seed()).  temp <= 0 is greedy (first index of the maximum)."""

    def __init__(self, state: int | None = None):
        lib = cuda_lib()
        self._state = ctypes.c_uint64(lib.dpuf_cuda_sample_seed() if state is None else state)

    @property
    def state(self) -> int:
        return int(self._state.value)

    def __call__(self, logits: np.ndarray, temp: float) -> int:
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        r = cuda_lib().dpuf_cuda_sample_token(lg.ctypes.data, lg.size, float(temp), ctypes.byref(self._state))
        if r < 0:
            raise ValueError("dpuf_cuda_sample_token: empty logits")
        return int(r)


def embed(blob, ids: np.ndarray) -> np.ndarray:
    lib = cuda_lib()
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty((len(ids), blob.cols), dtype=np.float32)
    lib.dpuf_embed_qr_hadamard4_packed_f32(len(ids), blob.cols, ids.ctypes.data, blob.tiles.ctypes.data,
                                           blob.tile_offsets.ctypes.data, blob.sign_bits.ctypes.data, out.ctypes.data)
    err = last_error()
    if err:
        raise RuntimeError(err)
    return out

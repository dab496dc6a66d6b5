"""Checkers for the CUDA engine.  TEST INFRASTRUCTURE ONLY: imported by tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs, never by the
product package.

Two CPU engines with the reference's C ABI are driven here:
  * OracleEngine - the scalar C restatement oracle/dpuf_oracle.c (liboracle.so, built by
    `build()` below from this directory);
  * RefEngine    - the reference's own AVX2/OpenMP engine compiled from its unmodified
    sources by oracle/build_ref.sh into oracle/_ref/libdpuf_avx2.so.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libdpuf_avx2.so"
# Where the reference sources are, for rebuilding oracle/_ref: env DPUF_REFERENCE_DIR (no default;
# without it an existing oracle/_ref build is kept as it is).
REF_SRC_ENV = "DPUF_REFERENCE_DIR"


def build(force: bool = False) -> pathlib.Path:
    src = HERE / "dpuf_oracle.c"
    hdr = HERE.parent / "include" / "dpuf_kernels.h"
    if force or not ORACLE_LIB.exists() or max(src.stat().st_mtime, hdr.stat().st_mtime) > ORACLE_LIB.stat().st_mtime:
        subprocess.run(["gcc", "-O2", "-std=gnu11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
                        "-fno-fast-math", str(src), "-o", str(ORACLE_LIB), "-lm"], check=True)
    return ORACLE_LIB


def build_ref(ref_dir: pathlib.Path | None = None) -> pathlib.Path | None:
    """Builds oracle/_ref/libdpuf_avx2.so from the reference sources at `ref_dir` (default: env
    DPUF_REFERENCE_DIR).  Without sources, an existing build is returned as it is (or None)."""
    if ref_dir is None and os.environ.get(REF_SRC_ENV):
        ref_dir = pathlib.Path(os.environ[REF_SRC_ENV])
    if ref_dir is None or not (ref_dir / "dpuf_engine.c").exists():
        return REF_LIB if REF_LIB.exists() else None
    subprocess.run(["bash", str(HERE / "build_ref.sh"), str(ref_dir)], check=True, capture_output=True)
    return REF_LIB


_F = ctypes.POINTER(ctypes.c_float)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_F)


class _EngineBase:
    lib: ctypes.CDLL

    def argmax(self, logits: np.ndarray) -> int:
        """First index of the maximum (greedy sample_token, dpuf-cli.c:1997-2005)."""
        return int(np.argmax(logits))  # numpy returns the first maximal index


class OracleEngine(_EngineBase):
    _lib = None

    @classmethod
    def lib_(cls) -> ctypes.CDLL:
        if cls._lib is None:
            if not ORACLE_LIB.exists():
                raise RuntimeError("oracle/liboracle.so is not built")
            lib = ctypes.CDLL(str(ORACLE_LIB))
            lib.orc_engine_create.restype = ctypes.c_void_p
            lib.orc_engine_create.argtypes = [ctypes.c_void_p] * 5
            lib.orc_engine_destroy.argtypes = [ctypes.c_void_p]
            lib.orc_engine_reset_cache.argtypes = [ctypes.c_void_p]
            lib.orc_engine_forward.restype = ctypes.c_int32
            lib.orc_engine_forward.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32,
                                               ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
            lib.orc_matmul_mode12_f32.argtypes = [ctypes.c_int32] * 4 + [ctypes.c_void_p] * 5
            lib.orc_embed_mode12_f32.argtypes = [ctypes.c_int32, ctypes.c_int32] + [ctypes.c_void_p] * 5
            lib.orc_prep_mode12.argtypes = [ctypes.c_int32] + [ctypes.c_void_p] * 5
            lib.orc_swiglu_is_vector.restype = ctypes.c_int32
            lib.orc_swiglu_is_vector.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]
            cls._lib = lib
        return cls._lib

    def __init__(self, model):
        self.lib = self.lib_()
        self.model = model
        self.h = self.lib.orc_engine_create(*model.create_args())
        if not self.h:
            raise RuntimeError("orc_engine_create failed")
        self.vocab = model.shape.vocab

    def close(self):
        if self.h:
            self.lib.orc_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def reset(self):
        self.lib.orc_engine_reset_cache(self.h)

    def forward(self, ids, pos0: int, only_last: int = 1, zone: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        M = len(ids)
        out = np.empty((1 if only_last == 1 else M, self.vocab), dtype=np.float32)
        zone_out = np.zeros(4, dtype=np.int32)
        rc = self.lib.orc_engine_forward(self.h, M, ids.ctypes.data, pos0, only_last,
                                         out.ctypes.data if only_last != 2 else None, zone_out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"orc_engine_forward -> {rc}")
        return (out, zone_out) if zone else out


class RefEngine(_EngineBase):
    """The reference engine (dpuf_engine.c) through its own C ABI (dpuf_kernels.h:316-360)."""
    _lib = None

    @classmethod
    def available(cls) -> bool:
        return REF_LIB.exists()

    @classmethod
    def lib_(cls) -> ctypes.CDLL:
        if cls._lib is None:
            if not REF_LIB.exists():
                raise RuntimeError("oracle/_ref/libdpuf_avx2.so is not built (needs the reference sources)")
            lib = ctypes.CDLL(str(REF_LIB))
            lib.dpuf_engine_create.restype = ctypes.c_void_p
            lib.dpuf_engine_create.argtypes = [ctypes.c_void_p] * 5
            lib.dpuf_engine_destroy.argtypes = [ctypes.c_void_p]
            lib.dpuf_engine_reset_cache.argtypes = [ctypes.c_void_p]
            lib.dpuf_engine_forward_batch.restype = ctypes.c_int32
            lib.dpuf_engine_forward_batch.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                                      ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
            lib.dpuf_matmul_qr_hadamard4_packed_f32.argtypes = [ctypes.c_int32] * 4 + [ctypes.c_void_p] * 5
            lib.dpuf_embed_qr_hadamard4_packed_f32.argtypes = [ctypes.c_int32, ctypes.c_int32] + [ctypes.c_void_p] * 5
            cls._lib = lib
        return cls._lib

    def __init__(self, model, n_threads: int = 8):
        self.lib = self.lib_()
        self.model = model
        # the engine runs min(n_threads, 32, omp_get_max_threads()) threads (dpuf_engine.c:1219-1223)
        self.threads = min(int(n_threads), 32, set_omp_threads(n_threads))
        model.cfg.n_threads = n_threads
        self.h = self.lib.dpuf_engine_create(*model.create_args())
        model.cfg.n_threads = 8
        if not self.h:
            raise RuntimeError("reference dpuf_engine_create failed")
        self.vocab = model.shape.vocab

    def close(self):
        if self.h:
            self.lib.dpuf_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def reset(self):
        self.lib.dpuf_engine_reset_cache(self.h)

    def forward(self, ids, pos0: int, only_last: int = 1):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        M = len(ids)
        out = np.empty((1 if only_last == 1 else M, self.vocab), dtype=np.float32)
        rc = self.lib.dpuf_engine_forward_batch(self.h, M, ids.ctypes.data, pos0, only_last,
                                                out.ctypes.data if only_last != 2 else None)
        if rc != 0:
            raise RuntimeError(f"reference forward -> {rc}")
        return out


def oracle_matmul(M, blob, x):
    """Standalone mode-12 matmul through the C restatement: out[M][rows]."""
    lib = OracleEngine.lib_()
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((M, blob.rows), dtype=np.float32)
    lib.orc_matmul_mode12_f32(M, blob.rows, blob.cols, blob.n_tiles, x.ctypes.data, blob.tiles.ctypes.data,
                              blob.tile_offsets.ctypes.data, blob.sign_bits.ctypes.data, out.ctypes.data)
    return out


def oracle_matmul_had(mode: int, M, blob, x):
    """Mode 13 (QR_HAD4_ASYM) or 14 (QR_HAD6) matmul restated (dpuf_avx2.c:3084-3144)."""
    lib = OracleEngine.lib_()
    lib.orc_matmul_had_asym_f32.argtypes = [ctypes.c_int32] * 5 + [ctypes.c_void_p] * 5
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((M, blob.rows), dtype=np.float32)
    lib.orc_matmul_had_asym_f32(int(mode == 14), M, blob.rows, blob.cols, blob.n_tiles, x.ctypes.data,
                                blob.tiles.ctypes.data, blob.tile_offsets.ctypes.data, blob.sign_bits.ctypes.data,
                                out.ctypes.data)
    return out


def oracle_embed_had(mode: int, blob, ids):
    """Mode 13 / 14 row lookup restated (dpuf_avx2.c:3146-3221): out[len(ids)][cols]."""
    lib = OracleEngine.lib_()
    lib.orc_embed_had_asym_f32.argtypes = [ctypes.c_int32] * 3 + [ctypes.c_void_p] * 5
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty((ids.size, blob.cols), dtype=np.float32)
    lib.orc_embed_had_asym_f32(int(mode == 14), ids.size, blob.cols, ids.ctypes.data, blob.tiles.ctypes.data,
                               blob.tile_offsets.ctypes.data, blob.sign_bits.ctypes.data, out.ctypes.data)
    return out


def ref_matmul(M, blob, x):
    lib = RefEngine.lib_()
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty((M, blob.rows), dtype=np.float32)
    lib.dpuf_matmul_qr_hadamard4_packed_f32(M, blob.rows, blob.cols, blob.n_tiles, x.ctypes.data,
                                            blob.tiles.ctypes.data, blob.tile_offsets.ctypes.data,
                                            blob.sign_bits.ctypes.data, out.ctypes.data)
    return out


def greedy_run(engine, prompt, n_decode: int):
    """pp(prompt) + n_decode greedy steps at batch 1 (run_turn_ex, dpuf-cli.c:2344-2420).
    Returns (generated ids, list of per-step logits [prefill last + each decode step])."""
    engine.reset()
    # prompts longer than the 256-token batch limit go in chunks, only the last one returning
    # logits (run_turn_ex, dpuf-cli.c:2380-2395)
    for c0 in range(0, len(prompt) - 256, 256):
        engine.forward(prompt[c0:c0 + 256], c0, 2)
    c0 = (len(prompt) - 1) // 256 * 256
    logits = [engine.forward(prompt[c0:], c0, 1)[0].copy()]
    ids = []
    pos = len(prompt)
    for _ in range(n_decode):
        nxt = int(np.argmax(logits[-1]))
        ids.append(nxt)
        logits.append(engine.forward(np.array([nxt], np.int32), pos, 1)[0].copy())
        pos += 1
    return ids, logits


def cpu_model_string() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def host_threads() -> int:
    """Host cores this process may run on (its CPU affinity)."""
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def set_omp_threads(n: int) -> int:
    """Sets the OpenMP thread count of the calling thread in the process's GNU OpenMP runtime
    (the libgomp.so.1 the reference library links) and returns omp_get_max_threads() as read
    back.  The reference engine clamps its team to omp_get_max_threads()
    (dpuf_engine.c:1219-1223), which launchers such as torchrun pin to 1 through
    OMP_NUM_THREADS; this call overrides that for the CPU baseline."""
    gomp = ctypes.CDLL("libgomp.so.1")
    gomp.omp_set_num_threads.argtypes = [ctypes.c_int]
    gomp.omp_get_max_threads.restype = ctypes.c_int
    gomp.omp_set_num_threads(int(n))
    return int(gomp.omp_get_max_threads())


def zone_a(logits: np.ndarray, za_tiles: int, margin: float):
    """Zone-A exit test and masking on one row of fp32 logits, as dpuf_engine.c:2101-2135:
    sequential top-2 with strict '>' over logits[0, min(16Z, V)) from -1e30, exit iff
    margin > 0 and (b1 - b2) >= margin in fp32; on exit logits[16Z, V) = -1e9.  Z is the
    already-clamped tile count.  Returns (exit, logits after masking, b1, b2)."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    n = min(za_tiles * 16, lg.size)
    b1 = b2 = np.float32(-1e30)
    for v in lg[:n].tolist():
        v = np.float32(v)
        if v > b1:
            b2, b1 = b1, v
        elif v > b2:
            b2 = v
    exit_ = bool(margin > 0.0 and np.float32(b1 - b2) >= np.float32(margin))
    if exit_:
        lg[za_tiles * 16:] = np.float32(-1e9)
    return exit_, lg, float(b1), float(b2)


REF_SAMPLE_LIB = HERE / "_ref" / "libdpuf_ref_sample.so"
SAMPLE_SEED = 88172645463325252  # initial g_rng, dpuf-cli.c:1987
_LIBM = None


def _expf(x: np.float32) -> np.float32:
    """The host's glibc expf (the reference calls libm's expf, dpuf-cli.c:2015)."""
    global _LIBM
    if _LIBM is None:
        _LIBM = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
        _LIBM.expf.restype = ctypes.c_float
        _LIBM.expf.argtypes = [ctypes.c_float]
    return np.float32(_LIBM.expf(float(x)))


def rand_f32(state: int) -> tuple[float, int]:
    """rand_f32 (dpuf-cli.c:1988-1995): one xorshift64 step of the state, then the top 24 bits
    of state * 2685821657736338717 (mod 2^64) / 2^24.  Returns (value, new state)."""
    m = (1 << 64) - 1
    x = state
    x ^= x >> 12
    x = (x ^ (x << 25)) & m
    x ^= x >> 27
    return float(np.float32(((x * 2685821657736338717) & m) >> 40) / np.float32(16777216.0)), x


def sample_token(logits: np.ndarray, temp: float, state: int) -> tuple[int, int]:
    """sample_token (dpuf-cli.c:1997-2027).  temp <= 0: first index of the maximum.  Else
    p_i = expf((l_i - max) * (1/temp)) in fp32, S their sequential double sum, r = u * S for
    one generator step u, and the first i whose sequential double prefix sum reaches r (V-1 if
    none).  np.cumsum is a sequential left-to-right accumulation.  Returns (id, new state)."""
    lg = np.asarray(logits, dtype=np.float32)
    t = np.float32(temp)
    if t <= 0:
        return int(np.argmax(lg)), state
    mx = lg.max()
    inv_t = np.float32(1.0) / t
    z = (lg - mx) * inv_t  # fp32, elementwise
    p = np.fromiter((_expf(v) for v in z.tolist()), dtype=np.float32, count=lg.size)
    cdf = np.cumsum(p.astype(np.float64))
    u, state = rand_f32(state)
    r = u * float(cdf[-1])
    hit = np.flatnonzero(cdf >= r)
    return (int(hit[0]) if hit.size else lg.size - 1), state


def ref_sample_token(logits: np.ndarray, temp: float, state: int) -> tuple[int, int]:
    """The reference CLI's own sample_token (oracle/_ref/libdpuf_ref_sample.so)."""
    lib = ctypes.CDLL(str(REF_SAMPLE_LIB))
    lib.ref_sample_token.restype = ctypes.c_int32
    lib.ref_sample_token.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p]
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    st = ctypes.c_uint64(state)
    r = lib.ref_sample_token(lg.ctypes.data, lg.size, float(temp), ctypes.byref(st))
    return int(r), int(st.value)


def expf_mismatch(bits0: int, got: np.ndarray) -> tuple[int, int]:
    """(count, first index) of the inputs bits0 .. bits0 + len(got) - 1 (float bit patterns) where
    `got` differs bit for bit from this host's libm expf (orc_expf_mismatch)."""
    lib = OracleEngine.lib_()
    lib.orc_expf_mismatch.restype = ctypes.c_int64
    lib.orc_expf_mismatch.argtypes = [ctypes.c_uint32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    got = np.ascontiguousarray(got, dtype=np.float32)
    first = ctypes.c_int64(-1)
    n = lib.orc_expf_mismatch(bits0, got.size, got.ctypes.data, ctypes.byref(first))
    return int(n), int(first.value)

"""Build and load the package's native libraries (all built in-tree, next to their sources).

libdpuf_pack.so  - host encoder for mode-12 blobs and the seeded weight generator (C, gcc).
libdpuf_cuda.so  - the CUDA engine and kernels behind the C ABI of include/dpuf_kernels.h
                   (nvcc, sm_100a only).

`load_*` never builds: a missing library is an error, so a GPU run can never fall back to
anything else.  `build_*` is called by `__graft_entry__.build()` and by developers.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import shutil
import subprocess

PKG_DIR = pathlib.Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"

PACK_LIB = PKG_DIR / "libdpuf_pack.so"
CUDA_LIB = PKG_DIR / "libdpuf_cuda.so"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CUDA_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CUDA_SOURCES = [
    "engine.cu",
    "expf_table.cu",
    "kernels_mode12.cu",
    "kernels_gemv.cu",
    "kernels_gemv_wg.cu",
    "kernels_gemm_tc.cu",
    "kernels_layer.cu",
    "kernels_attn.cu",
    "kernels_lmhead.cu",
    "kernels_decode.cu",
    "ops_abi.cu",
    "ops_had_asym.cu",
    "noalloc.cu",
    "sampling.cu",
]


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def _stale(target: pathlib.Path, sources: list[pathlib.Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def build_pack(force: bool = False) -> pathlib.Path:
    src = CSRC / "pack_mode12.c"
    if force or _stale(PACK_LIB, [src]):
        _run(["gcc", "-O3", "-std=gnu11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
              "-fno-fast-math", str(src), "-o", str(PACK_LIB), "-lm"])
    return PACK_LIB


def build_cuda(force: bool = False, extra: list[str] | None = None) -> pathlib.Path:
    srcs = [CSRC / s for s in CUDA_SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    if force or extra or _stale(CUDA_LIB, deps):
        objdir = PKG_DIR / "_build"
        objdir.mkdir(exist_ok=True)
        objs = []
        common = [NVCC, *CUDA_ARCH, "-O3", "-lineinfo", "-std=c++17", "--fmad=false",
                  "-Xcompiler", "-fPIC,-fvisibility=hidden,-ffp-contract=off", "-I", str(INCLUDE), "-I", str(CSRC),
                  "-Xptxas", "-warn-spills", *(extra or [])]
        for s in srcs:
            o = objdir / (s.stem + ".o")
            _run([*common, "-rdc=false", "-c", str(s), "-o", str(o)])
            objs.append(str(o))
        _run([NVCC, *CUDA_ARCH, "-shared", "-o", str(CUDA_LIB), *objs, "-lcuda", "-lcudart"])
    return CUDA_LIB


def _load(path: pathlib.Path, what: str) -> ctypes.CDLL:
    if not path.exists():
        raise RuntimeError(f"{what} is not built ({path}); run __graft_entry__.build() first")
    return ctypes.CDLL(str(path))


_pack = None
_cuda = None


def load_pack() -> ctypes.CDLL:
    global _pack
    if _pack is None:
        _pack = _load(PACK_LIB, "libdpuf_pack.so")
    return _pack


def load_cuda() -> ctypes.CDLL:
    global _cuda
    if _cuda is None:
        _cuda = _load(CUDA_LIB, "libdpuf_cuda.so")
    return _cuda

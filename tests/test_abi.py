"""The drop-in C ABI: libdpuf_cuda.so exports every symbol the headers declare, the struct
mirrors have the reference sizes, and without a GPU the engine refuses to start (no CPU path)."""
import ctypes
import pathlib
import re

import numpy as np
import pytest

from dpuf_b200 import _native, model as mdl

INCLUDE = pathlib.Path(__file__).resolve().parents[1] / "include"


def declared_symbols():
    names = set()
    for h in INCLUDE.glob("*.h"):
        text = h.read_text()
        for m in re.finditer(r"DPUF_EXPORT\s+[\w\s\*]+?\b(\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def cuda_lib():
    _native.build_cuda()
    return ctypes.CDLL(str(_native.CUDA_LIB))


def test_headers_declare_reference_engine_api():
    names = set(declared_symbols())
    ref_engine_api = {
        "dpuf_engine_create", "dpuf_engine_destroy", "dpuf_engine_reset_cache", "dpuf_engine_set_slot",
        "dpuf_engine_get_slot", "dpuf_engine_reset_slot", "dpuf_engine_slot_memory", "dpuf_engine_num_slots",
        "dpuf_engine_freeze_prefix", "dpuf_engine_apply_prefix", "dpuf_engine_get_prefix_len",
        "dpuf_engine_forward_batch", "dpuf_engine_forward_batch_ex", "dpuf_engine_forward_token",
        "dpuf_matmul_qr_hadamard4_packed_f32", "dpuf_embed_qr_hadamard4_packed_f32",
    }
    assert ref_engine_api <= names


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports_declared_symbol(cuda_lib, name):
    assert hasattr(cuda_lib, name), f"{name} declared in include/ but not exported"


def test_struct_sizes_match_reference():
    assert ctypes.sizeof(mdl.DpufWeightDesc) == 48
    assert ctypes.sizeof(mdl.DpufModelConfig) == 92
    assert ctypes.sizeof(mdl.DpufLayerWeights) == 368


def test_engine_without_gpu_fails_loudly(cuda_lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    from dpuf_b200 import engine

    m = mdl.SyntheticModel(mdl.TINY, seed=0)
    with pytest.raises(RuntimeError, match="dpuf_engine_create failed"):
        engine.CudaTransformerEngine(m)


def test_engine_rejects_non_mode12(cuda_lib):
    from dpuf_b200 import engine

    lib = engine.cuda_lib()
    m = mdl.SyntheticModel(mdl.TINY, seed=0)
    m.layers[0].w_q.mode = 10  # row-major Hadamard: not served by this engine
    assert not lib.dpuf_engine_create(*m.create_args())


def test_tp_entry_points_reject_bad_arguments(cuda_lib):
    """Tensor-parallel setup checks its arguments before touching a GPU."""
    from dpuf_b200 import engine

    lib = engine.cuda_lib()
    blob = np.zeros(engine.TP_BLOB_BYTES, np.uint8)
    assert lib.dpuf_cuda_tp_handle(None, 0, 2, blob.ctypes.data) == -1
    assert lib.dpuf_cuda_tp_attach(None, blob.ctypes.data) == -1
    with open(pathlib.Path(__file__).resolve().parents[1] / "include" / "dpuf_cuda.h") as f:
        assert f"#define DPUF_CUDA_TP_BLOB_BYTES {engine.TP_BLOB_BYTES}" in f.read()

"""Token sampling (scope row a13): the library's host sampler, the oracle's restatement and the
reference CLI's own sample_token (dpuf-cli.c:1987-2027, built from its source into
oracle/_ref/) pick the same ids and leave the same generator state.

The sampler is host code, so these run without a GPU."""
import ctypes

import numpy as np
import pytest

from dpuf_b200 import engine as eng
from oracle import oracle as orc

needs_ref = pytest.mark.skipif(not orc.REF_SAMPLE_LIB.exists(), reason="reference sampler not built")

TEMPS = [0.0, -1.0, 0.3, 0.7, 1.0, 1.5, 4.0]


def _logits(seed: int, V: int, kind: str) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return rng.normal(0.0, 3.0, V).astype(np.float32)
    if kind == "peaked":  # a few dominant ids, the rest far below (exp underflows to 0)
        lg = rng.normal(-80.0, 5.0, V).astype(np.float32)
        lg[rng.integers(0, V, 4)] = np.float32(10.0)
        return lg
    if kind == "ties":  # many equal maxima: greedy must return the first
        lg = rng.integers(-3, 3, V).astype(np.float32)
        return lg
    if kind == "masked":  # Zone-A masking leaves -1e9 after the zone
        lg = rng.normal(0.0, 2.0, V).astype(np.float32)
        lg[V // 3:] = np.float32(-1e9)
        return lg
    raise ValueError(kind)


def _draws(fn, lg, temp, n, state):
    ids = []
    for _ in range(n):
        i, state = fn(lg, temp, state)
        ids.append(i)
    return ids, state


def _lib_fn(lg, temp, state):
    st = ctypes.c_uint64(state)
    r = eng.cuda_lib().dpuf_cuda_sample_token(lg.ctypes.data, lg.size, float(temp), ctypes.byref(st))
    return int(r), int(st.value)


@needs_ref
@pytest.mark.parametrize("kind", ["normal", "peaked", "ties", "masked"])
@pytest.mark.parametrize("temp", TEMPS)
def test_library_sampler_matches_reference(kind, temp):
    lg = np.ascontiguousarray(_logits(7, 151936, kind))
    ref_ids, ref_state = _draws(orc.ref_sample_token, lg, temp, 6, orc.SAMPLE_SEED)
    got_ids, got_state = _draws(_lib_fn, lg, temp, 6, orc.SAMPLE_SEED)
    assert got_ids == ref_ids and got_state == ref_state


@needs_ref
@pytest.mark.parametrize("temp", [0.0, 0.5, 1.0])
def test_oracle_sampler_matches_reference(temp):
    for V, kind in [(1, "normal"), (17, "ties"), (4096, "peaked"), (20000, "normal")]:
        lg = np.ascontiguousarray(_logits(V, V, kind))
        assert _draws(orc.sample_token, lg, temp, 4, 12345) == _draws(orc.ref_sample_token, lg, temp, 4, 12345)


def test_library_sampler_matches_oracle_small():
    """Runs where the reference sources are absent too (the GPU box has only the oracle)."""
    for V, kind, temp in [(1, "normal", 0.8), (33, "ties", 0.0), (33, "ties", 2.0), (5000, "peaked", 1.0),
                          (5000, "normal", 0.6)]:
        lg = np.ascontiguousarray(_logits(V + 1, V, kind))
        assert _draws(_lib_fn, lg, temp, 5, orc.SAMPLE_SEED) == _draws(orc.sample_token, lg, temp, 5, orc.SAMPLE_SEED)


def test_sampler_object_and_errors():
    s = eng.Sampler()
    assert s.state == orc.SAMPLE_SEED == eng.cuda_lib().dpuf_cuda_sample_seed()
    lg = np.ascontiguousarray(_logits(3, 1000, "normal"))
    assert s(lg, 0.0) == int(np.argmax(lg)) and s.state == orc.SAMPLE_SEED  # greedy: no draw
    first = s(lg, 1.0)
    assert s.state != orc.SAMPLE_SEED
    assert first == orc.sample_token(lg, 1.0, orc.SAMPLE_SEED)[0]
    lib = eng.cuda_lib()
    assert lib.dpuf_cuda_sample_token(None, 10, ctypes.c_float(1.0), None) == -1
    assert lib.dpuf_cuda_sample_token(lg.ctypes.data, 0, ctypes.c_float(1.0), None) == -1
    assert lib.dpuf_cuda_sample_token(lg.ctypes.data, lg.size, ctypes.c_float(1.0), None) == -1
    with pytest.raises(ValueError):
        s(np.zeros(0, np.float32), 1.0)

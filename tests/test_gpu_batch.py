"""Batched serving (configuration 5 of the scope): one decode step for several independent
sequences, each in its own slot at its own position.  Every row must equal that sequence's own
batch-1 step (dpuf_engine_forward_token on its slot), which matches the reference engine (the
engine goldens in test_gpu_parity); so the batched step is bit-identical to the reference's
sequence-at-a-time decode."""
import numpy as np
import pytest

from _util import EnvScope, bitexact

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng_mod():
    from dpuf_b200 import engine

    return engine


@pytest.mark.parametrize("shape,n_seq", [("TINY", 5), ("TINY_MHA", 3), ("QWEN3_0_6B", 4)])
def test_decode_batch_matches_sequence_at_a_time(eng_mod, shape, n_seq):
    from dpuf_b200 import model as mdl

    m = mdl.SyntheticModel(getattr(mdl, shape), seed=6, norm_jitter=0.1)
    slots = [2 * i + 1 for i in range(n_seq)]  # not 0..n-1, and beyond the reference's 8
    prompts = [mdl.prompt_ids(5 + 7 * i, m.shape.vocab, 40 + i) for i in range(n_seq)]
    steps = 5
    with EnvScope([("DPUF_CUDA_SLOTS", "16")]):
        batched = eng_mod.CudaTransformerEngine(m)
        single = eng_mod.CudaTransformerEngine(m)
    try:
        assert batched.num_slots() == 16
        toks, pos = [], []
        for e in (batched, single):
            for sl, pr in zip(slots, prompts):
                assert e.set_slot(sl) == 0
                e.reset_slot(sl)
                lg = e.forward_batch(pr, 0)[0]
                if e is batched:
                    toks.append(int(np.argmax(lg)))
                    pos.append(len(pr))
        for _ in range(steps):
            nxt, logits = batched.decode_batch(slots, toks, pos, want_logits=True)
            for i, sl in enumerate(slots):
                assert single.set_slot(sl) == 0
                want = single.forward_token(toks[i], pos[i])
                assert bitexact(logits[i], want), (shape, i)
                assert int(nxt[i]) == int(np.argmax(want))
            toks = [int(t) for t in nxt]
            pos = [p + 1 for p in pos]
    finally:
        batched.close()
        single.close()


def test_decode_batch_rejects_bad_arguments(eng_mod):
    from dpuf_b200 import model as mdl

    m = mdl.SyntheticModel(mdl.TINY, seed=1)
    e = eng_mod.CudaTransformerEngine(m)
    try:
        lib = e.lib
        nxt = np.zeros(4, np.int32)
        ids = np.array([1, 2], np.int32)
        pos = np.array([0, 0], np.int32)
        dup = np.array([3, 3], np.int32)
        assert lib.dpuf_cuda_decode_batch(e._handle, 2, dup.ctypes.data, ids.ctypes.data, pos.ctypes.data,
                                          nxt.ctypes.data, None) == -1
        bad = np.array([0, 8], np.int32)  # default slot count is the reference's 8
        assert lib.dpuf_cuda_decode_batch(e._handle, 2, bad.ctypes.data, ids.ctypes.data, pos.ctypes.data,
                                          nxt.ctypes.data, None) == -1
        ok = np.array([0, 1], np.int32)
        far = np.array([0, m.shape.max_seq], np.int32)
        assert lib.dpuf_cuda_decode_batch(e._handle, 2, ok.ctypes.data, ids.ctypes.data, far.ctypes.data,
                                          nxt.ctypes.data, None) == -3
        assert lib.dpuf_cuda_decode_batch(e._handle, 0, ok.ctypes.data, ids.ctypes.data, pos.ctypes.data,
                                          nxt.ctypes.data, None) == -2
    finally:
        e.close()

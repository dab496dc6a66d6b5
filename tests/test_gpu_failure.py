"""Failure detection in the persistent decode kernel, without any GPU fault.

The reference's spin barrier waits for ever (dpuf_engine.c:53-92).  Every wait of the
persistent kernel is bounded instead: here the CTA computing the first q rows withholds them (the
engine's test hook "test_stall_unit"), so the waits on them run into a 20 ms limit ("wait_ms");
the kernel then sets its error word, every CTA stops waiting and returns, and forward_token
returns -6.  The next call on the same engine starts from a reset exchange area and must give
the reference's ids and logits bit for bit again."""
import numpy as np
import pytest

from _util import bitexact

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_engine_recovers():
    import torch

    from dpuf_b200 import engine, model as mdl
    from oracle import oracle as orc

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    m = mdl.SyntheticModel(mdl.TINY, seed=0, norm_jitter=0.1)
    prompt = mdl.prompt_ids(12, m.shape.vocab, 0)
    ref = orc.OracleEngine(m)
    want_ids, want_logits = orc.greedy_run(ref, prompt, 4)
    ref.close()

    e = engine.CudaTransformerEngine(m)
    assert e.persistent_decode()[0]
    e.set_option("wait_ms", 20)
    e.reset_cache()
    first = int(np.argmax(e.forward_batch(prompt, 0)[0]))
    e.set_option("test_stall_unit", 0)
    with pytest.raises(RuntimeError, match="rc=-6"):
        e.forward_token(first, len(prompt))
    assert "timed out" in engine.last_error()

    got_ids, got_logits = orc.greedy_run(e, prompt, 4)
    assert got_ids == want_ids
    for g, w in zip(got_logits, want_logits):
        assert bitexact(g, w)
    e.close()

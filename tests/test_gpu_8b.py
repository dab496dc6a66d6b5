"""The headline configuration: Qwen3-8B-shaped random-init model, pp32 then 32 greedy decode
steps at batch 1 (tg32), against the reference engine (oracle/_ref, built from the reference
sources) on the same host.  Ids and every step's logits must be bit-identical over the whole
generated sequence; both batch-1 paths (persistent kernel through forward_token, and the device
greedy loop) are checked."""
import numpy as np
import pytest

from _util import bitexact

pytestmark = pytest.mark.gpu


def test_8b_greedy_decode_matches_reference_engine():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dpuf_b200 import engine, model as mdl
    from oracle import oracle as orc

    if not orc.RefEngine.available():
        pytest.skip("oracle/_ref/libdpuf_avx2.so not built")
    m = mdl.SyntheticModel(mdl.QWEN3_8B, seed=0)
    prompt = mdl.prompt_ids(32, m.shape.vocab, 0)
    n = 32
    ref = orc.RefEngine(m, n_threads=8)
    want_ids, want_logits = orc.greedy_run(ref, prompt, n)
    ref.close()

    e = engine.CudaTransformerEngine(m)
    assert e.persistent_decode()[0]
    got_ids, got_logits = orc.greedy_run(e, prompt, n)
    assert got_ids == want_ids
    for g, w in zip(got_logits, want_logits):
        assert bitexact(g, w)
    e.reset_cache()
    first = int(np.argmax(e.forward_batch(prompt, 0)[0]))
    ids, _ = e.decode_greedy(first, len(prompt), n - 1)
    assert [first] + ids == want_ids
    e.close()

"""Configuration 4 at its full size: the Zone-A early exit on a 151936 x 4096 mode-12 LM head
(9496 tiles), Z = 1000 zone tiles (16,000 ids), margin 0.8, over 64 hidden vectors with a
planted dominant logit and 64 flat ones.  Exit decisions and greedy ids must equal the
reference's: its exported mode-12 matmul (the same per-row arithmetic as the engine's LM-head
tile range) followed by the restated exit test of dpuf_engine.c:2101-2135 (sequential top-2,
margin test, -1e9 masking of the rest, first-index argmax)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_zone_a_config4_size_matches_reference():
    import torch

    from dpuf_b200 import engine, packer
    from oracle import oracle as orc

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    rows, cols, za, margin = 151936, 4096, 1000, 0.8
    w = packer.gen_normal_bf16(41, 9, (rows, cols), 0.02)
    bv = packer.BlobView(packer.encode_mode12(w, "output.weight"))
    rng = np.random.default_rng(7)
    n_planted, n_flat = 64, 64
    planted = rng.integers(0, 16 * za, size=n_planted).astype(np.int32)
    x = rng.standard_normal((n_planted + n_flat, cols)).astype(np.float32)
    x[:n_planted] += np.float32(5.0) * engine.embed(bv, planted)
    ids, exits, _ = engine.zone_head(bv, x, za, margin)

    matmul = orc.ref_matmul if orc.RefEngine.available() else orc.oracle_matmul
    want_ids, want_exits = [], []
    for c0 in range(0, x.shape[0], 32):
        lg = matmul(min(32, x.shape[0] - c0), bv, x[c0:c0 + 32])
        for row in lg:
            ex, masked, _, _ = orc.zone_a(row, za, margin)
            want_exits.append(int(ex))
            want_ids.append(int(np.argmax(masked)))
    assert exits.tolist() == want_exits
    assert ids.tolist() == want_ids
    assert sum(want_exits[:n_planted]) >= n_planted // 2  # the planted half takes the exit path
    assert sum(want_exits[n_planted:]) <= n_flat // 2      # most flat vectors run the full vocabulary

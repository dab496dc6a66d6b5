"""dpuf_cuda_matmul_noalloc: the standalone mode-12 matmul for callers that cannot allocate
device memory (hosts that reserve the GPU's memory for their own pool at start-up, and loops
that cannot afford cudaMalloc's implicit synchronisation).  Its output must equal the
allocating entry point's (dpuf_matmul_qr_hadamard4_packed_f32) bit for bit - the tolerance of
every parity test here is zero - on two calls in a row, the second running over the scratch
array the first one left behind.  This file is collected last on purpose."""
import numpy as np
import pytest

from _util import bitexact, pack_case_blob

pytestmark = pytest.mark.gpu


def test_noalloc_matmul_matches_allocating_entry_point():
    import torch

    from dpuf_b200 import engine

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    lib = engine.cuda_lib()
    bv = pack_case_blob(3)  # 256 x 1024 mode-12 matrix
    # The caller owns every device buffer (allocated here by torch, not by the entry point).
    tiles = torch.from_numpy(bv.tiles.copy()).cuda()
    toff = torch.from_numpy(bv.tile_offsets.astype(np.uint64).view(np.int64).copy()).cuda()
    signs = torch.from_numpy(bv.sign_bits.copy()).cuda()
    # M = 300 crosses the 256-token chunk of the matmul; M = 1024 fills the 2^20-value array
    for call, M in enumerate((7, 1, 300, (1 << 20) // bv.cols)):
        x = np.random.default_rng(100 + call).standard_normal((M, bv.cols)).astype(np.float32)
        x[:, 128:160] = 0.0  # a zero block exercises the skipped-block path
        want = engine.matmul(M, bv, x)
        xd = torch.from_numpy(x).cuda()
        yd = torch.full((M, bv.rows), float("nan"), device="cuda")
        rc = lib.dpuf_cuda_matmul_noalloc(M, bv.rows, bv.cols, bv.n_tiles, xd.data_ptr(), tiles.data_ptr(),
                                          toff.data_ptr(), signs.data_ptr(), yd.data_ptr(), None)
        torch.cuda.synchronize()
        assert rc == 0, engine.last_error()
        assert bitexact(yd.cpu().numpy(), want), f"call {call} (M={M}) differs from the allocating entry point"


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch

    from dpuf_b200 import engine

    lib = engine.cuda_lib()
    bv = pack_case_blob(3)
    tiles = torch.from_numpy(bv.tiles.copy()).cuda()
    toff = torch.from_numpy(bv.tile_offsets.astype(np.uint64).view(np.int64).copy()).cuda()
    x = torch.zeros(1, device="cuda")
    y = torch.zeros(1, device="cuda")
    M = (1 << 20) // bv.cols + 1
    rc = lib.dpuf_cuda_matmul_noalloc(M, bv.rows, bv.cols, bv.n_tiles, x.data_ptr(), tiles.data_ptr(),
                                      toff.data_ptr(), None, y.data_ptr(), None)
    assert rc == -2
    assert "scratch" in engine.last_error()

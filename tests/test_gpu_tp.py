"""Tensor-parallel batch-1 decode (scope row e): two or four processes, one GPU each, split every
projection and the LM head of the persistent kernel between them and exchange outputs through
each other's memory.  Every rank must return the ids and logits of one GPU bit for bit (one
GPU matches the reference engine: test_gpu_parity / test_gpu_8b).

Needs as many GPUs as ranks; skipped otherwise."""
import os
import socket
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scenario(eng_mod, mdl, shape_name: str, seed: int, tp=None):
    """Prefill (M > 1, in full on every rank), three forward_token steps with logits, then a
    greedy run on the device; returns (ids, [logits...])."""
    m = mdl.SyntheticModel(mdl.SHAPES[shape_name], seed=seed, norm_jitter=0.1)
    e = eng_mod.CudaTransformerEngine(m, {"persistent": 1})
    try:
        on, why = e.persistent_decode()
        assert on, why
        if tp is not None:
            e.tp_attach(*tp)
        prompt = mdl.prompt_ids(9, m.shape.vocab, seed)
        e.reset_cache()
        logits = [e.forward_batch(prompt, 0)[0]]
        tok = int(np.argmax(logits[0]))
        pos = len(prompt)
        for _ in range(3):
            logits.append(e.forward_token(tok, pos))
            tok = int(np.argmax(logits[-1]))
            pos += 1
        ids, _ = e.decode_greedy(tok, pos, 20)
        last = np.empty(m.shape.vocab, np.float32)
        assert e.lib.dpuf_cuda_read_logits(e._handle, 0, last.ctypes.data) == 0
        logits.append(last)
        return ids, logits
    finally:
        e.close()


def _rank_main(rank: int, world: int, port: int, cases, out):
    import datetime

    import torch.distributed as dist

    os.environ["DPUF_CUDA_DEVICE"] = str(rank)
    sys.path.insert(0, REPO)
    from dpuf_b200 import engine as eng_mod
    from dpuf_b200 import model as mdl

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        for shape_name, seed in cases:
            dist.barrier()
            ids, logits = _scenario(eng_mod, mdl, shape_name, seed, (rank, world, eng_mod.torch_all_gather()))
            out.put((rank, shape_name, ids, [lg.tobytes() for lg in logits]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


CASES = [("tiny", 3), ("tiny-mha", 5), ("tiny-wide", 2), ("qwen3-0.6b", 0)]


@pytest.mark.parametrize("world", [2, 4])
def test_tp_decode_matches_one_gpu(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    sys.path.insert(0, REPO)
    from dpuf_b200 import engine as eng_mod
    from dpuf_b200 import model as mdl

    want = {name: _scenario(eng_mod, mdl, name, seed) for name, seed in CASES}
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, CASES, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=600) for _ in range(world * len(CASES))]
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for rank, name, ids, logits in got:
        w_ids, w_logits = want[name]
        assert ids == w_ids, (rank, name)
        assert len(logits) == len(w_logits)
        for a, b in zip(logits, w_logits):
            assert a == b.tobytes(), (rank, name)

"""The reference's own C host (dpuf-cli.c, unmodified) over this repository's containers and
engine library.

oracle/build_ref.sh links dpuf-cli.c twice: `dpuf-cli` over the reference engine and
`dpuf-cli-cuda` with libdpuf_cuda.so supplying every dpuf_engine_* symbol, as a user would
relink the CLI (the engine ABI of dpuf_kernels.h:316-360).  A greedy raw-mode turn
(run_turn_ex, dpuf-cli.c:2344-2420: `[tokens: ...]`, then the decoded continuation) must print
the same bytes from both.  The CPU case checks that the reference CLI reads the DPUF0001
container this repository writes (header, tensor index, model_config, tokenizer) and that its
greedy continuation is the oracle engine's.  Both run on a mode-12 model and on a hybrid one
(every matrix in mode 13 or 14, as the reference's had4p-hybrid packing assigns them).
"""
from __future__ import annotations

import pathlib
import subprocess

import numpy as np
import pytest

from dpuf_b200 import container

REPO = pathlib.Path(__file__).resolve().parents[1]
CLI_REF = REPO / "oracle" / "_ref" / "dpuf-cli"
CLI_CUDA = REPO / "oracle" / "_ref" / "dpuf-cli-cuda"
PROMPT = "Hello, B200! été"


def _render(ids, vocab_syms) -> bytes:
    """Bytes the CLI prints for generated ids under container.synthetic_tokenizer: the byte
    symbols decode to their byte, every other id to its literal "[id]" string."""
    inv = {s: b for b, s in enumerate(container.byte_symbols())}
    out = bytearray()
    for i in ids:
        s = vocab_syms[i]
        if i < 256:
            out.append(inv[s])
        else:
            out += s.encode("utf-8")
    return bytes(out)


def _turn(cli: pathlib.Path, model: pathlib.Path, n: int, threads: int = 4):
    r = subprocess.run([str(cli), "-m", str(model), "--raw", "--tokens", "-p", PROMPT, "-n", str(n),
                        "--temp", "0", "-t", str(threads)], capture_output=True, timeout=600)
    assert r.returncode == 0, r.stderr.decode(errors="replace")[-2000:]
    out = r.stdout
    lines = out.split(b"\n")
    tok_line = next(l for l in lines if l.startswith(b"[tokens:"))
    body = out.split(tok_line + b"\n", 1)[1]
    gen = body.split(b"\n\n[stats:", 1)[0]
    return tok_line, gen


@pytest.fixture(scope="module", params=[False, True], ids=["mode12", "hybrid"])
def tiny_file(tmp_path_factory, request):
    p = tmp_path_factory.mktemp("cli") / "tiny.dpuf"
    container.write_synthetic(p, "tiny", seed=11, hybrid=request.param)
    return p


def test_reference_cli_reads_container(tiny_file):
    if not CLI_REF.exists():
        pytest.skip("oracle/_ref/dpuf-cli is not built (needs the reference sources)")
    from oracle import oracle as orc

    n = 24
    tok_line, gen = _turn(CLI_REF, tiny_file, n)
    prompt = list(PROMPT.encode("utf-8"))
    assert tok_line == ("[tokens: " + " ".join(map(str, prompt)) + "]").encode()
    f = container.DpufFile(tiny_file)
    try:
        eng = orc.RefEngine(f, n_threads=4)
        try:
            ids, _ = orc.greedy_run(eng, np.array(prompt, np.int32), n)
        finally:
            eng.close()
        syms = f.meta["tokenizer"]["vocab"]
    finally:
        f.close()
    assert gen == _render(ids, syms)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,seed,n,hybrid", [("tiny", 11, 40, False), ("tiny-long", 5, 64, False),
                                                 ("tiny", 11, 40, True)])
def test_cli_relinked_on_cuda_engine(tmp_path, shape, seed, n, hybrid):
    """The reference CLI relinked on libdpuf_cuda.so prints what it prints on the reference
    engine (prompt ids and the greedy continuation, byte for byte)."""
    if not (CLI_REF.exists() and CLI_CUDA.exists()):
        pytest.skip("oracle/_ref/dpuf-cli{,-cuda} are not built (needs the reference sources)")
    p = tmp_path / f"{shape}.dpuf"
    container.write_synthetic(p, shape, seed=seed, hybrid=hybrid)
    ref = _turn(CLI_REF, p, n, threads=8)
    got = _turn(CLI_CUDA, p, n, threads=8)
    assert got[0] == ref[0]
    assert got[1] == ref[1]

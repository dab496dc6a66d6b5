"""GPU parity: the CUDA engine and ops, called through the C ABI, against the reference's
golden outputs and the CPU oracle.  Integer/byte work and every fp32 result are compared bit
for bit (the reference's operation order is reproduced), so the tolerance is zero."""
import numpy as np
import pytest

import scenarios as sc
from _util import EnvScope, bitexact, golden_arrays, golden_engine, pack_case_blob, run_scenario

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng_mod():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dpuf_b200 import _native, engine

    _native.build_cuda()
    engine.cuda_lib()
    return engine


@pytest.mark.parametrize("ci,M,kind", sc.MATMUL_CASES)
def test_matmul_matches_reference(eng_mod, ci, M, kind):
    bv = pack_case_blob(ci)
    x = sc.matmul_input(ci, M, kind, bv.cols)
    got = eng_mod.matmul(M, bv, x)
    assert bitexact(got, golden_arrays("matmul.npz")[f"matmul_{ci}_{M}_{kind}"])


@pytest.mark.parametrize("ci", [3, 4])
def test_embed_matches_reference(eng_mod, ci):
    g = golden_arrays("matmul.npz")
    bv = pack_case_blob(ci)
    assert bitexact(eng_mod.embed(bv, g[f"embed_{ci}_ids"]), g[f"embed_{ci}"])


@pytest.mark.parametrize("variant", ["0", "1", "2", "3"])
def test_expanded_gemm_shapes_match_oracle(eng_mod, variant):
    """Every shape of the expanded-weight GEMM (8 / 16 / 32 / 64 tokens per CTA, forced through
    env DPUF_CUDA_X8_VARIANT) on a 512x4096 matrix at M = 64: several stages per CTA with the
    ring reused, the scalar and the packed chains, against the oracle."""
    from dpuf_b200 import packer
    from oracle import oracle as orc

    w = packer.gen_normal_bf16(77, 5, (512, 4096), 0.02)
    bv = packer.BlobView(packer.encode_mode12(w, "blk.0.ffn_up.weight"))
    x = np.random.default_rng(77).standard_normal((64, 4096)).astype(np.float32)
    x[:, 64:96] = 0.0
    x[5, :] = 0.0
    with EnvScope([("DPUF_CUDA_X8_VARIANT", variant)]):
        assert bitexact(eng_mod.matmul(64, bv, x), orc.oracle_matmul(64, bv, x))


@pytest.mark.parametrize("expand", ["1", "0"])
@pytest.mark.parametrize("M", [1, 2, 5, 16, 17, 33, 64, 100, 256])
def test_matmul_token_counts_match_oracle(eng_mod, M, expand):
    """M > 1 runs on the tensor cores: over the expanded s8 copy of the matrix, or (env
    DPUF_CUDA_TC_EXPAND=0) unpacking the tiles in the kernel."""
    from oracle import oracle as orc

    bv = pack_case_blob(3)
    x = np.random.default_rng(M).standard_normal((M, bv.cols)).astype(np.float32)
    x[:, 64:96] = 0.0
    with EnvScope([("DPUF_CUDA_TC_EXPAND", expand)]):
        assert bitexact(eng_mod.matmul(M, bv, x), orc.oracle_matmul(M, bv, x))


@pytest.mark.parametrize("scn", sc.ENGINE_SCENARIOS, ids=lambda s: s.name)
def test_engine_matches_reference(eng_mod, scn):
    g = golden_engine()[scn.name]
    rec, logits, _ = run_scenario(eng_mod.CudaTransformerEngine, scn)
    assert rec["ids"] == g["ids"]
    assert rec["digests"] == g["digests"]
    if scn.all_logits:
        assert rec["prefill_all_digest"] == g["prefill_all_digest"]
    if scn.full_logits:
        assert bitexact(np.stack(logits), golden_arrays("engine_logits.npz")[scn.name])
    if "zone_exit" in g:
        za = max(256, int(dict(scn.env)["DPUF_EARLY_TILES"]))
        assert [bool(np.all(l[16 * za:] == np.float32(-1e9))) for l in logits] == g["zone_exit"]


def test_engine_without_graphs_or_pdl_matches(eng_mod):
    scn = sc.ENGINE_SCENARIOS[0]
    g = golden_engine()[scn.name]
    for opts in ({"graphs": 0}, {"pdl": 0}, {"persistent": 0}):
        rec, _, _ = run_scenario(lambda m: eng_mod.CudaTransformerEngine(m, opts), scn)
        assert rec["digests"] == g["digests"], opts
    with EnvScope([("DPUF_CUDA_TC_EXPAND", "0")]):  # the tensor-core GEMM unpacking in the kernel
        rec, _, _ = run_scenario(eng_mod.CudaTransformerEngine, scn)
    assert rec["digests"] == g["digests"]


def test_greedy_api_matches_logits(eng_mod):
    from dpuf_b200 import model as mdl

    m = mdl.SyntheticModel(mdl.TINY, seed=5, norm_jitter=0.1)
    e = eng_mod.CudaTransformerEngine(m)
    prompt = mdl.prompt_ids(9, m.shape.vocab, 5)
    e.reset_cache()
    lg = e.forward_batch(prompt, 0)[0]
    e.reset_cache()
    assert e.forward_greedy(prompt, 0) == int(np.argmax(lg))
    e.close()


@pytest.mark.parametrize("kv_type", [0, 1])
def test_slots_and_prefixes_match_oracle(eng_mod, kv_type):
    """Prefix freeze/apply and slot switching (dpuf_engine.c:1404-1600) give the same logits as
    recomputing the prefix, with the fp32 and the Q8 cache."""
    from dpuf_b200 import model as mdl
    from oracle import oracle as orc

    m = mdl.SyntheticModel(mdl.TINY, seed=2, norm_jitter=0.1)
    m.cfg.kv_type = kv_type
    e = eng_mod.CudaTransformerEngine(m)
    o = orc.OracleEngine(m)
    prefix = mdl.prompt_ids(12, m.shape.vocab, 2)
    tail = mdl.prompt_ids(5, m.shape.vocab, 9)
    e.reset_cache()
    e.forward_batch(prefix, 0)
    assert e.freeze_prefix(1, len(prefix)) == 1
    assert e.get_prefix_len(1) == len(prefix)
    assert e.set_slot(3) == 0 and e.get_slot() == 3
    assert e.apply_prefix(3, 1) == len(prefix)
    got = e.forward_batch(tail, len(prefix))[0]
    o.reset()
    o.forward(prefix, 0)
    want = o.forward(tail, len(prefix))[0]
    assert bitexact(got, want)
    # slot 0 still holds the prefix only; a fresh slot 5 starts empty
    assert e.set_slot(5) == 0
    e.reset_cache()
    got5 = e.forward_batch(tail, 0)[0]
    o.reset()
    assert bitexact(got5, o.forward(tail, 0)[0])
    assert e.num_slots() == 8 and e.slot_memory() > 0
    assert e.set_slot(8) == -1
    e.close()
    o.close()


def test_forward_error_codes(eng_mod):
    from dpuf_b200 import model as mdl

    m = mdl.SyntheticModel(mdl.TINY, seed=0)
    e = eng_mod.CudaTransformerEngine(m)
    lib = e.lib
    ids = np.zeros(300, np.int32)
    out = np.zeros(m.shape.vocab, np.float32)
    assert lib.dpuf_engine_forward_batch(e._handle, 0, ids.ctypes.data, 0, 1, out.ctypes.data) == -2
    assert lib.dpuf_engine_forward_batch(e._handle, 257, ids.ctypes.data, 0, 1, out.ctypes.data) == -2
    assert lib.dpuf_engine_forward_batch(e._handle, 4, ids.ctypes.data, m.shape.max_seq - 3, 1,
                                         out.ctypes.data) == -3
    assert lib.dpuf_engine_forward_batch(e._handle, 4, None, 0, 1, out.ctypes.data) == -1
    assert lib.dpuf_engine_forward_batch(e._handle, 4, ids.ctypes.data, 0, 1, None) == -1
    assert lib.dpuf_engine_forward_batch(e._handle, 4, ids.ctypes.data, 0, 2, None) == 0
    e.close()


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1040, 12288), (6144, 4096)])
def test_gemv_decode_shapes_match_oracle(eng_mod, rows, cols):
    """Decode GEMV on the 8B projection shapes: many stages per 16-row unit, so units are split
    between CTAs and finished by the last part to arrive; results stay bit-exact."""
    from dpuf_b200 import packer
    from oracle import oracle as orc

    w = packer.gen_normal_bf16(rows, cols, (rows, cols), 0.02)
    bv = packer.BlobView(packer.encode_mode12(w, f"shape{rows}x{cols}"))
    x = np.random.default_rng(rows + cols).standard_normal((1, cols)).astype(np.float32)
    x[:, 1024:1088] = 0.0
    want = orc.oracle_matmul(1, bv, x)
    for _ in range(2):  # the split arrival counters must be left at zero for the next call
        assert bitexact(eng_mod.matmul(1, bv, x), want)


@pytest.mark.parametrize("shape", ["TINY", "TINY_MHA", "TINY_WIDE"])
def test_persistent_decode_matches_step_kernels(eng_mod, shape):
    """Greedy decode as one persistent kernel gives the ids and last logits of the per-step
    kernels, which match the reference (the engine goldens above)."""
    from dpuf_b200 import model as mdl

    m = mdl.SyntheticModel(getattr(mdl, shape), seed=3, norm_jitter=0.1)
    prompt = mdl.prompt_ids(11, m.shape.vocab, 3)
    runs = []
    for persistent in (1, 0):
        e = eng_mod.CudaTransformerEngine(m, {"persistent": persistent})
        on, why = e.persistent_decode()
        assert on == bool(persistent), why
        e.reset_cache()
        first = int(np.argmax(e.forward_batch(prompt, 0)[0]))
        ids, _ = e.decode_greedy(first, len(prompt), 24)
        logits = np.empty(m.shape.vocab, np.float32)
        assert e.lib.dpuf_cuda_read_logits(e._handle, 0, logits.ctypes.data) == 0
        runs.append((ids, logits))
        e.close()
    assert runs[0][0] == runs[1][0]
    assert bitexact(runs[0][1], runs[1][1])


def test_persistent_decode_with_pruned_down(eng_mod):
    """DPUF_GEN_KEEP_TILES: rows beyond the kept down-projection tiles add zero to the residual."""
    from dpuf_b200 import model as mdl

    m = mdl.SyntheticModel(mdl.TINY, seed=4, norm_jitter=0.1)
    prompt = mdl.prompt_ids(7, m.shape.vocab, 4)
    outs = []
    with EnvScope([("DPUF_GEN_KEEP_TILES", "12")]):
        for persistent in (1, 0):
            e = eng_mod.CudaTransformerEngine(m, {"persistent": persistent})
            e.reset_cache()
            e.forward_batch(prompt, 0)
            outs.append([e.forward_token(t, len(prompt) + i) for i, t in enumerate((5, 17, 300))])
            e.close()
    for a, b in zip(*outs):
        assert bitexact(a, b)


def test_zone_head_matches_oracle(eng_mod):
    """Zone-A LM head (config 4 semantics) on planted and flat hidden vectors: exit decisions and
    greedy ids equal the oracle's (mode-12 matmul + the reference's sequential top-2 test)."""
    from dpuf_b200 import packer
    from oracle import oracle as orc

    rows, cols, za, margin = 40960, 512, 1000, 0.8
    w = packer.gen_normal_bf16(21, 7, (rows, cols), 0.02)
    bv = packer.BlobView(packer.encode_mode12(w, "output.weight"))
    rng = np.random.default_rng(4)
    planted = rng.integers(0, 16 * za, size=4).astype(np.int32)
    x = rng.standard_normal((8, cols)).astype(np.float32)
    x[:4] += np.float32(20.0) * eng_mod.embed(bv, planted)
    ids, exits, _ = eng_mod.zone_head(bv, x, za, margin)
    want_ids, want_exits = [], []
    for i in range(x.shape[0]):
        lg = orc.oracle_matmul(1, bv, x[i:i + 1])[0]
        ex, masked, _, _ = orc.zone_a(lg, za, margin)
        want_exits.append(int(ex))
        want_ids.append(int(np.argmax(masked)))
    assert exits.tolist() == want_exits
    assert ids.tolist() == want_ids
    assert 0 < sum(want_exits) < len(want_exits)  # both paths exercised
    assert ids[:4].tolist() == planted.tolist()


@pytest.mark.parametrize("rows,cols,name", [(12288, 4096, "blk.0.mlp_in"), (4096, 12288, "blk.0.ffn_down.weight")])
@pytest.mark.parametrize("M", [1, 32])
def test_config2_ops_match_oracle(eng_mod, rows, cols, name, M):
    """The isolated-op configuration: gate-shaped and down-shaped matrices at M = 1 and 32; the
    down-shaped input is dead-zoned like a SwiGLU output."""
    from dpuf_b200 import packer
    from oracle import oracle as orc

    w = packer.gen_normal_bf16(31, rows, (rows, cols), 0.02)
    bv = packer.BlobView(packer.encode_mode12(w, name))
    x = np.random.default_rng(M).standard_normal((M, cols)).astype(np.float32)
    if "down" in name:
        x[np.abs(x) < 0.3] = 0.0
    assert bitexact(eng_mod.matmul(M, bv, x), orc.oracle_matmul(M, bv, x))


def test_q8_cache_layout_and_fallback(eng_mod):
    """kv_type 1 stores hd int8 values + hd/32 fp32 scales per row: a slot takes the bytes the
    reference's dpuf_engine_slot_memory reports (dpuf_engine.c:1476-1488), and decode runs on
    the per-step kernels (the persistent kernel keeps the fp32 cache)."""
    from dpuf_b200 import model as mdl

    m = mdl.SyntheticModel(mdl.QWEN3_0_6B, seed=1)
    m.cfg.kv_type = 1
    e = eng_mod.CudaTransformerEngine(m)
    try:
        s = m.shape
        elems = s.layers * s.max_seq * s.n_kv * s.head_dim
        assert e.slot_memory() == 2 * elems + 2 * (elems // 32) * 4
        on, why = e.persistent_decode()
        assert not on and "Q8" in why
        ids, _ = e.decode_greedy(5, 0, 4)
        assert len(ids) == 4
    finally:
        e.close()


def test_embeds_in_matches_reference(eng_mod):
    """forward_batch_ex with embeds_in (dpuf_engine.c:1658-1672): every row from the caller's
    embeddings, then greedy steps from ids; and a mixed call whose ids -1 take their rows from
    embeds_in; DeepStack rows added after layers 0 and 2 (dpuf_engine.c:2046-2054), for 12 rows
    and for one token.  Logits equal the reference engine's (digests in engine.json)."""
    import ctypes

    from dpuf_b200 import model as mdl

    g = golden_engine()["embeds_in"]
    shape, seed, rows = sc.EMBEDS_CASE
    m = mdl.SyntheticModel(mdl.SHAPES[shape], seed=seed, norm_jitter=0.1)
    e = eng_mod.CudaTransformerEngine(m)
    try:
        f = e.lib.dpuf_engine_forward_batch_ex
        f.restype = ctypes.c_int32
        f.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p] + \
            [ctypes.c_void_p] * 4 + [ctypes.c_int32, ctypes.c_void_p]
        emb = sc.embeds_input(rows, m.shape.hidden)
        V = m.shape.vocab
        e.reset_cache()
        allp = np.empty((rows, V), np.float32)
        assert f(e._handle, rows, None, 0, emb.ctypes.data, None, None, None, None, 0, allp.ctypes.data) == 0
        assert sc.logits_digest(allp) == g["all_digest"]
        tok, pos = int(np.argmax(allp[-1])), rows
        for dig, want in zip(g["steps_digests"], g["steps_ids"]):
            lg = e.forward_token(tok, pos)
            assert sc.logits_digest(lg) == dig
            tok = int(np.argmax(lg))
            assert tok == want
            pos += 1
        e.reset_cache()
        mixed = mdl.prompt_ids(rows, V, seed).astype(np.int32)
        mixed[list(sc.EMBEDS_MIXED_NEG)] = -1
        last = np.empty((1, V), np.float32)
        assert f(e._handle, rows, mixed.ctypes.data, 0, emb.ctypes.data, None, None, None, None, 1,
                 last.ctypes.data) == 0
        assert sc.logits_digest(last) == g["mixed_last_digest"]
        ds = sc.deepstack_input(rows, m.shape.hidden)
        e.reset_cache()
        arr = (ctypes.c_void_p * 3)(ds[0].ctypes.data, None, ds[2].ctypes.data)
        assert f(e._handle, rows, None, 0, emb.ctypes.data, None, None, None, arr, 0, allp.ctypes.data) == 0
        assert sc.logits_digest(allp) == g["deepstack_all_digest"]
        one = np.array([int(np.argmax(allp[-1]))], np.int32)
        arr1 = (ctypes.c_void_p * 3)(ds[1].ctypes.data, ds[0].ctypes.data, None)
        assert f(e._handle, 1, one.ctypes.data, rows, None, None, None, None, arr1, 1, last.ctypes.data) == 0
        assert sc.logits_digest(last) == g["deepstack_token_digest"]
        # a negative id without embeddings
        assert f(e._handle, rows, mixed.ctypes.data, 0, None, None, None, None, None, 1, last.ctypes.data) == -1
    finally:
        e.close()


def test_rope_positions_match_reference(eng_mod):
    """forward_batch_ex rotary positions (dpuf_engine.c:1679-1696): pos_t shifted from the cache
    position on a model without M-RoPE; M-RoPE t/h/w rows (the reference's own cos/sin
    formula, eng_compute_mrope_cos_sin) for 12 tokens and for one token, and equal t/h/w (the
    tables' row).  Logits equal the reference engine's."""
    import ctypes

    from dpuf_b200 import model as mdl

    g = golden_engine()["rope_positions"]
    shape, seed, rows = sc.EMBEDS_CASE
    for mrope in (0, 1):
        m = mdl.SyntheticModel(mdl.SHAPES[shape], seed=seed, norm_jitter=0.1)
        if mrope:
            m.cfg.has_mrope = 1
            for i, v in enumerate(sc.MROPE_SECTION):
                m.cfg.mrope_section[i] = v
        e = eng_mod.CudaTransformerEngine(m)
        try:
            f = e.lib.dpuf_engine_forward_batch_ex
            f.restype = ctypes.c_int32
            f.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p] + \
                [ctypes.c_void_p] * 4 + [ctypes.c_int32, ctypes.c_void_p]
            V = m.shape.vocab
            ids = mdl.prompt_ids(rows, V, seed).astype(np.int32)
            allp = np.empty((rows, V), np.float32)
            last = np.empty((1, V), np.float32)
            e.reset_cache()
            if not mrope:
                pt = (np.arange(rows) + 5).astype(np.int32)
                assert f(e._handle, rows, ids.ctypes.data, 0, None, pt.ctypes.data, None, None, None, 0,
                         allp.ctypes.data) == 0
                assert sc.logits_digest(allp) == g["shifted_all_digest"]
                far = np.full(rows, m.shape.max_seq, np.int32)
                assert f(e._handle, rows, ids.ctypes.data, 0, None, far.ctypes.data, None, None, None, 1,
                         last.ctypes.data) == -3
                continue
            t, h, w = sc.rope_positions(rows)
            assert f(e._handle, rows, ids.ctypes.data, 0, None, t.ctypes.data, h.ctypes.data, w.ctypes.data, None, 0,
                     allp.ctypes.data) == 0
            assert sc.logits_digest(allp) == g["mrope_all_digest"]
            one = np.array([int(np.argmax(allp[-1]))], np.int32)
            t1, h1, w1 = (np.array([v], np.int32) for v in (rows, 2, 7))
            assert f(e._handle, 1, one.ctypes.data, rows, None, t1.ctypes.data, h1.ctypes.data, w1.ctypes.data, None,
                     1, last.ctypes.data) == 0
            assert sc.logits_digest(last) == g["mrope_token_digest"]
            e1 = np.array([rows + 1], np.int32)
            assert f(e._handle, 1, one.ctypes.data, rows + 1, None, e1.ctypes.data, e1.ctypes.data, e1.ctypes.data,
                     None, 1, last.ctypes.data) == 0
            assert sc.logits_digest(last) == g["mrope_equal_digest"]
        finally:
            e.close()


def test_hybrid_model_runs_on_step_kernels(eng_mod):
    """A model with mode-13/14 layers (the reference's had4p-hybrid packing) is served by the
    per-step kernels - batch-1 steps included, bit-identical to the oracle engine - and the
    engine says why it does not use the persistent kernel."""
    from dpuf_b200 import model as mdl
    from oracle import oracle as orc

    m = mdl.SyntheticModel(mdl.TINY_G3, seed=9, norm_jitter=0.1, hybrid=True)
    prompt = mdl.prompt_ids(23, m.shape.vocab, 9)
    ref = orc.OracleEngine(m)
    want_ids, want_logits = orc.greedy_run(ref, prompt, 6)
    ref.close()
    e = eng_mod.CudaTransformerEngine(m)
    on, why = e.persistent_decode()
    assert not on and "mode-13/14" in why
    got_ids, got_logits = orc.greedy_run(e, prompt, 6)
    assert got_ids == want_ids
    assert all(bitexact(g, w) for g, w in zip(got_logits, want_logits))
    e.reset_cache()
    e.forward_batch(prompt, 0)
    ids, _ = e.decode_greedy(want_ids[0], len(prompt), 5)
    assert ids == want_ids[1:6]
    e.close()

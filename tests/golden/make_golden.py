"""Generates the golden fixtures in this directory from the REFERENCE itself.

Run in a container that has the reference sources:
    python tests/golden/make_golden.py REF_DIR      (or env DPUF_REFERENCE_DIR)
    python tests/golden/make_golden.py REF_DIR --scenario NAME[,NAME]   (only those engine
                                                                         scenarios, merged)
It builds oracle/_ref/libdpuf_avx2.so from the unmodified reference sources
(oracle/build_ref.sh), imports the reference packer module, and records:
  * pack.json     sha256 of the reference packer's blob for each PACK_CASES input;
  * matmul.npz    outputs of the reference's exported dpuf_matmul_qr_hadamard4_packed_f32 and
                  dpuf_embed_qr_hadamard4_packed_f32;
  * engine.json / engine_logits.npz
                  greedy ids and logit digests (full logits for small vocabularies) of the
                  reference engine (8 threads) for every ENGINE_SCENARIOS entry.
The engine models are packed with this repository's packer, whose bytes are checked against
the reference packer by pack.json.
"""
from __future__ import annotations

import ctypes
import json
import os
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from dpuf_b200 import _native, model as mdl, packer  # noqa: E402
from oracle import oracle as orc  # noqa: E402
import scenarios as sc  # noqa: E402


def main() -> None:
    args = sys.argv[1:]
    only = None
    if "--scenario" in args:  # --scenario NAME[,NAME...]: only those engine scenarios
        i = args.index("--scenario")
        only = args[i + 1].split(",")
        del args[i:i + 2]
    src = args[0] if args else os.environ.get(orc.REF_SRC_ENV, "")
    if not src:
        raise SystemExit("give the reference source directory (argument or DPUF_REFERENCE_DIR)")
    ref_dir = pathlib.Path(src)
    _native.build_pack()
    orc.build_ref(ref_dir)
    if only:
        update_scenarios(only)
        return
    sys.path.insert(0, str(ref_dir))
    import dpuf_format as ref_format  # the reference packer module

    # ---- packer
    pack = {}
    blobs = []
    for i, (rows, cols, name, seed) in enumerate(sc.PACK_CASES):
        w = packer.gen_normal_bf16(seed, i, (rows, cols), 0.02)
        w[0, :32] = 0
        w[min(1, rows - 1), 5] = packer.fp32_to_bf16(np.array([3.0], np.float32))[0]
        ref_blob = ref_format.encode_tensor_qr_hadamard4_packed(w, tensor_name=name)
        pack[f"case{i}"] = {"rows": rows, "cols": cols, "name": name, "seed": seed, "sha256": sc.blob_digest(ref_blob)}
        blobs.append(packer.BlobView(np.frombuffer(ref_blob, dtype=np.uint8).copy()))
    (HERE / "pack.json").write_text(json.dumps(pack, indent=1))

    # ---- standalone ops
    arrays = {}
    for ci, M, kind in sc.MATMUL_CASES:
        bv = blobs[ci]
        x = sc.matmul_input(ci, M, kind, bv.cols)
        arrays[f"matmul_{ci}_{M}_{kind}"] = orc.ref_matmul(M, bv, x)
    lib = orc.RefEngine.lib_()
    for ci in (3, 4):
        bv = blobs[ci]
        ids = np.random.default_rng(ci).integers(0, bv.rows, size=9).astype(np.int32)
        out = np.empty((len(ids), bv.cols), np.float32)
        lib.dpuf_embed_qr_hadamard4_packed_f32(len(ids), bv.cols, ids.ctypes.data, bv.tiles.ctypes.data,
                                               bv.tile_offsets.ctypes.data, bv.sign_bits.ctypes.data, out.ctypes.data)
        arrays[f"embed_{ci}_ids"] = ids
        arrays[f"embed_{ci}"] = out
    np.savez_compressed(HERE / "matmul.npz", **arrays)

    # ---- modes 13 / 14 (blobs from the reference packer, outputs from the reference library)
    had = {}
    for ci, (rows, cols, mode, seed) in enumerate(sc.HAD_CASES):
        w = packer.gen_normal_bf16(seed, 100 + ci, (rows, cols), 0.02)
        enc = ref_format.encode_tensor_qr_had4_asym if mode == 13 else ref_format.encode_tensor_qr_had6
        had[f"blob_{ci}"] = np.frombuffer(enc(w, tensor_name=f"had.{ci}"), np.uint8).copy()
    fn = {13: lib.dpuf_matmul_qr_had4_asym_f32, 14: lib.dpuf_matmul_qr_had6_f32}
    for f in fn.values():
        f.argtypes = [ctypes.c_int32] * 4 + [ctypes.c_void_p] * 5
    for ci, M, kind in sc.HAD_MATMUL:
        rows, cols, mode, _ = sc.HAD_CASES[ci]
        bv = packer.BlobView(had[f"blob_{ci}"])
        assert bv.mode == mode
        x = sc.matmul_input(50 + ci, M, kind, cols)
        out = np.empty((M, rows), np.float32)
        fn[mode](M, rows, cols, bv.n_tiles, x.ctypes.data, bv.tiles.ctypes.data, bv.tile_offsets.ctypes.data,
                 bv.sign_bits.ctypes.data, out.ctypes.data)
        had[f"out_{ci}_{M}_{kind}"] = out
    emb = {13: lib.dpuf_embed_qr_had4_asym_f32, 14: lib.dpuf_embed_qr_had6_f32}
    for f in emb.values():
        f.argtypes = [ctypes.c_int32] * 2 + [ctypes.c_void_p] * 5
    for ci, (rows, cols, mode, _) in enumerate(sc.HAD_CASES):
        bv = packer.BlobView(had[f"blob_{ci}"])
        ids = sc.had_embed_ids(ci, rows)
        out = np.empty((ids.size, cols), np.float32)
        emb[mode](ids.size, cols, ids.ctypes.data, bv.tiles.ctypes.data, bv.tile_offsets.ctypes.data,
                  bv.sign_bits.ctypes.data, out.ctypes.data)
        had[f"embed_{ci}"] = out
    np.savez_compressed(HERE / "had_asym.npz", **had)

    # ---- engine scenarios
    eng_out = {}
    eng_logits = {}
    for s in sc.ENGINE_SCENARIOS:
        rec, full = scenario_golden(s)
        eng_out[s.name] = rec
        if full is not None:
            eng_logits[s.name] = full
    eng_out["embeds_in"] = embeds_golden(lib)
    eng_out["rope_positions"] = rope_golden(lib)
    (HERE / "engine.json").write_text(json.dumps(eng_out, indent=1))
    np.savez_compressed(HERE / "engine_logits.npz", **eng_logits)


def scenario_golden(s):
    """Greedy ids and logit digests of one engine scenario on the reference engine (8 threads);
    returns (record, full logits or None)."""
    saved = {k: os.environ.get(k) for k, _ in s.env}
    os.environ.update(dict(s.env))
    try:
        m = mdl.SyntheticModel(mdl.SHAPES[s.shape], seed=s.seed, norm_jitter=s.norm_jitter, hybrid=s.hybrid)
        m.cfg.kv_type = s.kv_type
        ref = orc.RefEngine(m, n_threads=8)
        prompt = mdl.prompt_ids(s.prompt_len, m.shape.vocab, s.seed)
        rec = {"prompt": prompt.tolist()}
        if s.all_logits:
            ref.reset()
            allp = ref.forward(prompt, 0, 0)
            rec["prefill_all_digest"] = sc.logits_digest(allp)
        ids, logits = orc.greedy_run(ref, prompt, s.n_decode)
        rec["ids"] = ids
        rec["digests"] = [sc.logits_digest(l) for l in logits]
        rec["head"] = [l[:4].tolist() for l in logits]
        rms = float(np.sqrt(np.mean(np.stack(logits) ** 2)))
        rec["logit_rms"] = rms
        if dict(s.env).get("DPUF_EARLY_TILES"):
            za = max(256, int(dict(s.env)["DPUF_EARLY_TILES"]))
            rec["zone_exit"] = [bool(np.all(l[16 * za:] == np.float32(-1e9))) for l in logits]
        ref.close()
        print(s.name, "ids", ids[:8], "rms", rms, flush=True)
        return rec, (np.stack(logits) if s.full_logits else None)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def update_scenarios(names) -> None:
    """(Re)computes only the named engine scenarios and merges them into engine.json."""
    path = HERE / "engine.json"
    eng_out = json.loads(path.read_text())
    logits_path = HERE / "engine_logits.npz"
    eng_logits = dict(np.load(logits_path)) if logits_path.exists() else {}
    for s in sc.ENGINE_SCENARIOS:
        if s.name in names:
            rec, full = scenario_golden(s)
            if full is not None:
                eng_logits[s.name] = full
            eng_out[s.name] = rec
    path.write_text(json.dumps(eng_out, indent=1))
    np.savez_compressed(logits_path, **eng_logits)


def embeds_golden(lib) -> dict:
    """forward_batch_ex with embeds_in on the reference engine (8 threads): all rows from
    embeddings (every row's logits), then 4 greedy steps from ids; and a mixed call whose ids
    -1 take their rows from embeds_in (last row's logits)."""
    shape, seed, rows = sc.EMBEDS_CASE
    m = mdl.SyntheticModel(mdl.SHAPES[shape], seed=seed, norm_jitter=0.1)
    ref = orc.RefEngine(m, n_threads=8)
    f = lib.dpuf_engine_forward_batch_ex
    f.restype = ctypes.c_int32
    f.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p] + \
        [ctypes.c_void_p] * 4 + [ctypes.c_int32, ctypes.c_void_p]
    emb = sc.embeds_input(rows, m.shape.hidden)
    V = m.shape.vocab
    ref.reset()
    allp = np.empty((rows, V), np.float32)
    assert f(ref.h, rows, None, 0, emb.ctypes.data, None, None, None, None, 0, allp.ctypes.data) == 0
    rec = {"all_digest": sc.logits_digest(allp)}
    tok, pos, digs, ids = int(np.argmax(allp[-1])), rows, [], []
    for _ in range(4):
        lg = ref.forward(np.array([tok], np.int32), pos, 1)[0]
        digs.append(sc.logits_digest(lg))
        tok = int(np.argmax(lg))
        ids.append(tok)
        pos += 1
    rec["steps_digests"], rec["steps_ids"] = digs, ids
    ref.reset()
    mixed = mdl.prompt_ids(rows, V, seed).astype(np.int32)
    mixed[list(sc.EMBEDS_MIXED_NEG)] = -1
    last = np.empty((1, V), np.float32)
    assert f(ref.h, rows, mixed.ctypes.data, 0, emb.ctypes.data, None, None, None, None, 1, last.ctypes.data) == 0
    rec["mixed_last_digest"] = sc.logits_digest(last)
    # DeepStack rows for layers 0 and 2 (layer 1: none) with embeddings, all rows' logits; then
    # one token from an id with DeepStack rows.  The reference adds the DeepStack rows right
    # after each thread's own part of the down projection, without a barrier
    # (dpuf_engine.c:2018-2054), so with several threads a row may be added to before another
    # thread has written it and the result depends on timing (repeated 8-thread runs differ).
    # One thread cannot race; for this model its SwiGLU split and down-projection path give the
    # same bits as eight threads (the digests above match either way).
    ref.close()
    ref = orc.RefEngine(m, n_threads=1)
    ds = sc.deepstack_input(rows, m.shape.hidden)
    ref.reset()
    arr = (ctypes.c_void_p * 3)(ds[0].ctypes.data, None, ds[2].ctypes.data)
    assert f(ref.h, rows, None, 0, emb.ctypes.data, None, None, None, arr, 0, allp.ctypes.data) == 0
    rec["deepstack_all_digest"] = sc.logits_digest(allp)
    one = np.array([int(np.argmax(allp[-1]))], np.int32)
    arr1 = (ctypes.c_void_p * 3)(ds[1].ctypes.data, ds[0].ctypes.data, None)
    assert f(ref.h, 1, one.ctypes.data, rows, None, None, None, None, arr1, 1, last.ctypes.data) == 0
    rec["deepstack_token_digest"] = sc.logits_digest(last)
    ref.close()
    return rec


def rope_golden(lib) -> dict:
    """forward_batch_ex rotary positions (dpuf_engine.c:1679-1696): pos_t = pos0 + m + 5 on a
    model without M-RoPE; on an M-RoPE model (sections MROPE_SECTION) distinct t/h/w rows, then a
    one-token call with distinct and one with equal t/h/w.  Reference engine, 8 threads."""
    shape, seed, rows = sc.EMBEDS_CASE
    f = lib.dpuf_engine_forward_batch_ex
    f.restype = ctypes.c_int32
    f.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p] + \
        [ctypes.c_void_p] * 4 + [ctypes.c_int32, ctypes.c_void_p]
    rec = {}
    for mrope in (0, 1):
        m = mdl.SyntheticModel(mdl.SHAPES[shape], seed=seed, norm_jitter=0.1)
        if mrope:
            m.cfg.has_mrope = 1
            for i, v in enumerate(sc.MROPE_SECTION):
                m.cfg.mrope_section[i] = v
        ref = orc.RefEngine(m, n_threads=8)
        V = m.shape.vocab
        ids = mdl.prompt_ids(rows, V, seed).astype(np.int32)
        allp = np.empty((rows, V), np.float32)
        last = np.empty((1, V), np.float32)
        ref.reset()
        if not mrope:
            pt = (np.arange(rows) + 5).astype(np.int32)
            assert f(ref.h, rows, ids.ctypes.data, 0, None, pt.ctypes.data, None, None, None, 0, allp.ctypes.data) == 0
            rec["shifted_all_digest"] = sc.logits_digest(allp)
        else:
            t, h, w = sc.rope_positions(rows)
            assert f(ref.h, rows, ids.ctypes.data, 0, None, t.ctypes.data, h.ctypes.data, w.ctypes.data, None, 0,
                     allp.ctypes.data) == 0
            rec["mrope_all_digest"] = sc.logits_digest(allp)
            one = np.array([int(np.argmax(allp[-1]))], np.int32)
            t1, h1, w1 = (np.array([v], np.int32) for v in (rows, 2, 7))
            assert f(ref.h, 1, one.ctypes.data, rows, None, t1.ctypes.data, h1.ctypes.data, w1.ctypes.data, None, 1,
                     last.ctypes.data) == 0
            rec["mrope_token_digest"] = sc.logits_digest(last)
            e1 = np.array([rows + 1], np.int32)
            assert f(ref.h, 1, one.ctypes.data, rows + 1, None, e1.ctypes.data, e1.ctypes.data, e1.ctypes.data, None,
                     1, last.ctypes.data) == 0
            rec["mrope_equal_digest"] = sc.logits_digest(last)
        ref.close()
    return rec


if __name__ == "__main__":
    main()

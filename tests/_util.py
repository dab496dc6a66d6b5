"""Helpers shared by the parity tests."""
from __future__ import annotations

import json
import os
import pathlib

import numpy as np

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def golden_engine() -> dict:
    return json.loads((GOLDEN / "engine.json").read_text())


def golden_pack() -> dict:
    return json.loads((GOLDEN / "pack.json").read_text())


def golden_arrays(name: str):
    return np.load(GOLDEN / name)


def bitexact(a, b) -> bool:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def pack_case_blob(i: int):
    """The PACK_CASES[i] matrix encoded by this repository's packer (same input as make_golden)."""
    import scenarios as sc
    from dpuf_b200 import packer

    rows, cols, name, seed = sc.PACK_CASES[i]
    w = packer.gen_normal_bf16(seed, i, (rows, cols), 0.02)
    w[0, :32] = 0
    w[min(1, rows - 1), 5] = packer.fp32_to_bf16(np.array([3.0], np.float32))[0]
    return packer.BlobView(packer.encode_mode12(w, name))


class EnvScope:
    def __init__(self, pairs):
        self.pairs = list(pairs)
        self.saved = {}

    def __enter__(self):
        for k, v in self.pairs:
            self.saved[k] = os.environ.get(k)
            os.environ[k] = v
        return self

    def __exit__(self, *exc):
        for k, v in self.saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def run_scenario(engine_factory, scenario):
    """Builds the scenario's model, runs prompt + greedy decode on the engine made by
    engine_factory(model); returns (record dict, list of logits)."""
    import scenarios as sc
    from dpuf_b200 import model as mdl
    from oracle import oracle as orc

    with EnvScope(scenario.env):
        m = mdl.SyntheticModel(mdl.SHAPES[scenario.shape], seed=scenario.seed, norm_jitter=scenario.norm_jitter,
                               hybrid=scenario.hybrid)
        m.cfg.kv_type = scenario.kv_type
        eng = engine_factory(m)
        try:
            prompt = mdl.prompt_ids(scenario.prompt_len, m.shape.vocab, scenario.seed)
            rec = {"prompt": prompt.tolist()}
            if scenario.all_logits:
                eng.reset()
                rec["prefill_all_digest"] = sc.logits_digest(eng.forward(prompt, 0, 0))
            ids, logits = orc.greedy_run(eng, prompt, scenario.n_decode)
            rec["ids"] = ids
            rec["digests"] = [sc.logits_digest(l) for l in logits]
            return rec, logits, m
        finally:
            eng.close()

"""Shared helpers of the model-level tests: a random-init model of a configuration, its forward on
the oracle (the restated WASM executor, f32) and on the CUDA backend (plan mode and ragged bulk
mode), and the parity metrics of the BASELINE acceptance rules (cosine, max abs difference,
argmax)."""
from __future__ import annotations

import numpy as np

from kleinhirn_b200.encoder import mask_and_types, packed_inputs, word_rows
from kleinhirn_b200.plan import build_plan
from kleinhirn_b200.spec import output_cols, spec_from_hf_config
from kleinhirn_b200.synthetic import random_weights, to_f16
from oracle import host


class Model:
    def __init__(self, config: dict, extras: dict, seed: int = 0, f16: bool = False):
        self.spec, self.head, _ = spec_from_hf_config(config, extras)
        w32 = random_weights(self.spec, self.head, seed=seed)
        self.f16 = f16
        # the f16 manifest's values; the oracle runs them in f32 (the WASM path is f32 only)
        self.weights = to_f16(w32) if f16 else w32
        self.weights32 = {k: v.astype(np.float32) for k, v in self.weights.items()}
        self.cols = output_cols(self.spec, self.head)

    @property
    def word_table(self) -> np.ndarray:
        return self.weights["embeddings.word.weight"]


def oracle_forward(m: Model, id_lists, length: int, threads: int = 1) -> np.ndarray:
    """One B = 1 call per sequence on the bucket plan (src/encoder.ts:348-375), f32."""
    plan = build_plan(m.spec, m.head, length, 1, 0, False)
    rt = host.Runtime(threads=threads)
    try:
        host.load_weights(rt, m.weights32, [plan])
        p = rt.plan(plan)
        table = m.weights32["embeddings.word.weight"]
        outs = []
        for ids in id_lists:
            inputs = [{"inputIds": list(ids)}]
            mask, types = mask_and_types(m.spec, inputs, length)
            p.upload(word_rows(table, inputs, length), mask, types)
            p.run(len(ids))
            o = p.read_output()
            outs.append(o[: len(ids) * m.cols] if m.head["type"] == "token" else o[: m.cols])
        return np.stack(outs) if m.head["type"] != "token" else outs
    finally:
        rt.close()


def cuda_forward_plan(backend, m: Model, id_lists, length: int) -> np.ndarray:
    """The same B = 1 calls through the CUDA backend's PlanRunner."""
    plan = build_plan(m.spec, m.head, length, 1, 0, m.f16)
    r = backend.runner(plan)
    outs = []
    for ids in id_lists:
        inputs = [{"inputIds": list(ids)}]
        mask, types = mask_and_types(m.spec, inputs, length)
        r.upload(word_rows(m.word_table, inputs, length), mask, types)
        r.run(len(ids))
        o = r.read_output()
        outs.append(o[: len(ids) * m.cols] if m.head["type"] == "token" else o[: m.cols])
    r.destroy()
    return np.stack(outs) if m.head["type"] != "token" else outs


def cuda_forward_bulk(backend, m: Model, id_lists, length: int, chunk_tokens: int = 4096) -> np.ndarray:
    plan = build_plan(m.spec, m.head, length, 1, 0, m.f16)
    r = backend.runner(plan)
    emb, types, lens = packed_inputs(m.spec, m.word_table, [np.asarray(x) for x in id_lists])
    bulk = backend.bulk(r, int(lens.sum()), len(lens), chunk_tokens)
    out = bulk.run_batch(lens, emb, types if "typeIds" in plan["inputs"] else None)
    bulk.close()
    r.destroy()
    if m.head["type"] == "token":  # one row per packed token: split per sequence
        ends = np.cumsum(lens)
        return [out[e - n: e].ravel() for e, n in zip(ends, lens)]
    return out


def cosine_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.asarray(a, dtype=np.float64).reshape(len(a), -1)
    b = np.asarray(b, dtype=np.float64).reshape(len(b), -1)
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1) + 1e-30)

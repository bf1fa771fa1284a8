"""Host-side packing of encoder inputs and the calls a user makes.

Restates the parts of ``EncoderModel`` (src/encoder.ts) that sit in front of the Backend seam:

- ``mask_and_types`` = ``maskAndTypes`` (src/encoder.ts:284-314): prefix mask, type ids and,
  for RoBERTa / XLM-R, the position row packed in the high 16 bits (positionRows,
  src/plan/spec.ts:63-66).
- ``word_rows``      = ``wordRows`` (src/encoder.ts:273-282) with the host word table
  (``FullTable.copyRow``, src/words.ts:43-49): rows past a sequence's end stay zero.
- ``next_batch_size`` / ``batch_stride`` = src/cache.ts:14-19 / :81-83.
- ``Encoder.run_ids`` / ``run_ids_batch`` = src/encoder.ts:348-375 / :461-474 over a backend's
  PlanRunner; ``Encoder.run_ragged`` packs any number of sequences back to back for the
  CUDA backend's bulk path (no padding rows, src/encoder.ts:439-448 pads them).

Tokenisation stays upstream (inputs are token ids, as in the reference's runIds).
"""
from __future__ import annotations

import numpy as np

from .plan import build_plan
from .spec import output_cols, position_rows

BATCH_SIZES = (1, 4, 8, 16)
MAX_BATCH = 16


def next_batch_size(n: int) -> int:
    """src/cache.ts:14-19."""
    for b in BATCH_SIZES:
        if n <= b:
            return b
    raise ValueError(f"batch of {n} exceeds the maximum of {MAX_BATCH}")


def batch_stride(max_seq_len: int) -> int:
    """src/cache.ts:81-83."""
    return -(-max_seq_len // 64) * 64


def mask_and_types(spec: dict, inputs: list[dict], length: int) -> tuple[np.ndarray, np.ndarray]:
    """src/encoder.ts:284-314. Each input: {"inputIds": [...], "typeIds": [...] (optional)}."""
    n = len(inputs)
    mask = np.zeros(length * n, dtype=np.float32)
    type_ids = np.zeros(length * n, dtype=np.uint32)
    emb = spec["embed"]
    for b, inp in enumerate(inputs):
        ids = inp["inputIds"]
        mask[b * length: b * length + len(ids)] = 1
        if inp.get("typeIds") is not None and emb["typeVocab"] > 0:
            for i in range(len(ids)):
                t = inp["typeIds"][i] if i < len(inp["typeIds"]) else 0
                if not isinstance(t, (int, np.integer)) or t < 0 or t >= emb["typeVocab"]:
                    raise ValueError(f"token type {t} is not an integer inside the {emb['typeVocab']} type rows")
                type_ids[b * length + i] = t
        pad = emb.get("padId")
        if pad is not None:
            rows = position_rows(pad, [int(x) for x in ids])
            for i in range(length):
                p = rows[i] if i < len(rows) else pad
                if p >= emb["maxPositions"] or p > 0xFFFF:
                    raise ValueError(f"position row {p} of id {i} is outside the {emb['maxPositions']} position rows")
                type_ids[b * length + i] |= np.uint32(p << 16)
    return mask, type_ids


def word_rows(table: np.ndarray, inputs: list[dict], length: int) -> np.ndarray:
    """src/encoder.ts:273-282: word rows of sequence b at row b * length; rows past a
    sequence's end stay zero. `table` is [vocab, E] in the storage type."""
    width = table.shape[1]
    out = np.zeros((length * len(inputs), width), dtype=table.dtype)
    for b, inp in enumerate(inputs):
        ids = np.asarray(inp["inputIds"], dtype=np.int64)
        if ids.size and (ids.min() < 0 or ids.max() >= table.shape[0]):
            raise ValueError(f"token id outside the vocabulary of {table.shape[0]} rows")
        out[b * length: b * length + ids.size] = table[ids]
    return out


def packed_inputs(spec: dict, table: np.ndarray, id_lists: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Ragged packing for the bulk path: word rows and type ids of every sequence back to back
    (each sequence's rows exactly as mask_and_types / word_rows give them at B = 1)."""
    lens = np.array([len(x) for x in id_lists], dtype=np.int32)
    ids = np.concatenate([np.asarray(x, dtype=np.int64) for x in id_lists]) if id_lists else np.zeros(0, np.int64)
    if ids.size and (ids.min() < 0 or ids.max() >= table.shape[0]):
        raise ValueError(f"token id outside the vocabulary of {table.shape[0]} rows")
    emb = table[ids]
    types = np.zeros(ids.size, dtype=np.uint32)
    pad = spec["embed"].get("padId")
    if pad is not None:
        # positionRows per sequence: pad ids keep row pad, others pad + running count
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
        not_pad = (ids != pad).astype(np.int64)
        csum = np.cumsum(not_pad)
        base = np.repeat(np.concatenate([[0], csum])[starts], lens)
        rows = np.where(not_pad == 1, pad + (csum - base), pad)
        if rows.size and rows.max() >= spec["embed"]["maxPositions"]:
            raise ValueError("position row outside the position table")
        types |= (rows.astype(np.uint32) << np.uint32(16))
    return emb, types, lens


class Encoder:
    """The calls of EncoderModel over one backend, for the encoder heads (classify, token,
    embed): run_ids (B = 1 on the smallest bucket), run_ids_batch (sorted, chunks of 16 at a
    64-row stride), run_ragged (the CUDA backend's bulk path)."""

    def __init__(self, backend, spec: dict, head: dict, word_table: np.ndarray, buckets=(128, 512),
                 f16: bool = True):
        self.backend = backend
        self.spec = spec
        self.head = head
        self.words = word_table
        self.f16 = f16
        self.cols = output_cols(spec, head)
        self.plans = {}
        for L in buckets:
            plan = build_plan(spec, head, L, 1, 0, f16)
            backend.check(plan)
            self.plans[L] = backend.runner(plan)
        self.batch_plans = {}
        self._bulk = None

    def check_positions(self, seq_len: int) -> None:
        """src/encoder.ts:340-346."""
        e = self.spec["embed"]
        if seq_len > e["maxPositions"] - e["positionOffset"]:
            raise ValueError(f"input of {seq_len} tokens exceeds the {e['maxPositions']} position rows "
                             f"minus offset {e['positionOffset']}")

    def pick_bucket(self, seq_len: int):
        fits = sorted((L for L in self.plans if seq_len <= L))
        if not fits:
            raise ValueError(f"seqLen {seq_len} exceeds the loaded buckets")
        return self.plans[fits[0]]

    def _shape(self, data: np.ndarray, b: int, seq_len: int, runner) -> np.ndarray:
        cols = self.cols
        if self.head["type"] == "token":
            start = b * runner.length * cols
            return data[start: start + seq_len * cols].reshape(seq_len, cols)
        return data[b * cols: (b + 1) * cols]

    def run_ids(self, ids) -> np.ndarray:
        """src/encoder.ts:348-375."""
        seq_len = len(ids)
        if seq_len == 0:
            raise ValueError("empty input")
        self.check_positions(seq_len)
        runner = self.pick_bucket(seq_len)
        inputs = [{"inputIds": ids}]
        mask, types = mask_and_types(self.spec, inputs, runner.length)
        runner.upload(word_rows(self.words, inputs, runner.length), mask, types)
        runner.run(seq_len)
        out = self._shape(runner.read_output(), 0, seq_len, runner)
        if not np.all(np.isfinite(out)):
            raise FloatingPointError("engine output: values are not finite")
        return out

    def _batch_plan(self, stride: int, batch: int):
        key = (stride, batch)
        if key not in self.batch_plans:
            plan = self.backend.fit_batch(lambda b: build_plan(self.spec, self.head, stride, b, 0, self.f16), batch)
            self.batch_plans[key] = self.backend.runner(plan) if plan else None
        return self.batch_plans[key]

    def run_ids_batch(self, id_lists) -> list[np.ndarray]:
        """src/encoder.ts:461-474 with runChunk / submitPiece (src/encoder.ts:407-448)."""
        for i, ids in enumerate(id_lists):
            if len(ids) == 0:
                raise ValueError(f"empty input (input {i})")
        order = sorted(range(len(id_lists)), key=lambda i: (len(id_lists[i]), i))
        results: list = [None] * len(id_lists)
        for start in range(0, len(order), MAX_BATCH):
            idx = order[start: start + MAX_BATCH]
            inputs = [{"inputIds": id_lists[i]} for i in idx]
            max_seq = max(len(x["inputIds"]) for x in inputs)
            self.check_positions(max_seq)
            plan = self.pick_bucket(max_seq)
            n = next_batch_size(len(inputs))
            stride = min(plan.length, batch_stride(max_seq))
            bplan = (self._batch_plan(stride, n) if n > 1 else None) or plan
            out = []
            while len(out) < len(inputs):
                rows_in = inputs[len(out): len(out) + bplan.batch]
                padded = rows_in + [{"inputIds": []}] * (bplan.batch - len(rows_in))
                rows = max(len(x["inputIds"]) for x in rows_in) if bplan.batch == 1 else bplan.length * bplan.batch
                mask, types = mask_and_types(self.spec, padded, bplan.length)
                bplan.upload(word_rows(self.words, padded, bplan.length), mask, types)
                bplan.run(rows)
                data = bplan.read_output()
                out.extend(self._shape(data, i, len(x["inputIds"]), bplan) for i, x in enumerate(rows_in))
            for i, o in zip(idx, out):
                results[i] = o
        return results

    def run_ragged(self, id_lists, chunk_tokens: int = 65536) -> np.ndarray:
        """Every sequence through the CUDA backend's bulk path in one call: [n, cols] outputs in
        input order (pooled heads)."""
        lens = [len(x) for x in id_lists]
        if not lens or min(lens) == 0:
            raise ValueError("empty input")
        self.check_positions(max(lens))
        L = max(self.plans)
        emb, types, lens_a = packed_inputs(self.spec, self.words, id_lists)
        bulk = self.backend.bulk(self.plans[L], int(lens_a.sum()), len(lens), chunk_tokens)
        try:
            return bulk.run_batch(lens_a, emb, types)
        finally:
            bulk.close()

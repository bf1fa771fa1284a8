"""Model-level parity of the CUDA backend with the oracle, through the C ABI.

Acceptance rules: f32 plans give identical argmax and cosine >= 0.9999
against the oracle; f16 plans give cosine >= 0.999 and outputs within 2e-2 absolute (scaled by
max(1, |output|)) against the oracle run in f32 on the same f16 weights. Ragged bulk runs give
the B = 1 results of every sequence."""
import json
from pathlib import Path

import numpy as np
import pytest

from harness import Model, cosine_rows, cuda_forward_bulk, cuda_forward_plan, oracle_forward
from kleinhirn_b200 import synthetic

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "forward_golden.json").read_text())
F16_ABS = 2e-2


@pytest.fixture(scope="module")
def backend_factory():
    from kleinhirn_b200.backend import CudaBackend
    made = []

    def make(m):
        be = CudaBackend(m.weights)
        made.append(be)
        return be
    yield make
    for b in made:
        b.dispose()


def per_item(fn):
    """Token heads give one array per sequence (rows x classes, flattened): compare item by item."""
    def check(got, want):
        if isinstance(got, list) or isinstance(want, list):
            assert len(got) == len(want)
            for g, w in zip(got, want):
                fn(np.asarray(g, dtype=np.float64)[None, :], np.asarray(w, dtype=np.float64)[None, :])
        else:
            fn(got, want)
    return check


@per_item
def assert_f32(got, want):
    cos = cosine_rows(got, want)
    assert cos.min() >= 0.9999, cos
    if want.shape[1] > 1:
        assert np.array_equal(np.argmax(got, 1), np.argmax(want, 1))


@per_item
def assert_f16(got, want):
    cos = cosine_rows(got, want)
    assert cos.min() >= 0.999, cos
    scale = max(1.0, float(np.abs(want).max()))
    assert np.abs(got - want).max() <= F16_ABS * scale, np.abs(got - want).max()


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
@pytest.mark.parametrize("f16", [False, True], ids=["f32", "f16"])
def test_family_parity_plan_and_bulk(case, f16, backend_factory):
    m = Model(case["config"], case["extras"], seed=case["seed"], f16=f16)
    be = backend_factory(m)
    ids = [it["ids"] for it in case["items"]]
    want = oracle_forward(m, ids, 32)
    got = cuda_forward_plan(be, m, ids, 32)
    (assert_f16 if f16 else assert_f32)(got, want)
    if not f16:
        # the reference's own float64 forward, through the golden file
        for g, it in zip(got, case["items"]):
            w = np.array(it["want"])
            g = np.asarray(g, dtype=np.float64).ravel()
            assert g @ w / (np.linalg.norm(g) * np.linalg.norm(w)) >= 0.9999
    # ragged packing changes which keys share a 128-key tile, so the online softmax may round P
    # differently: equal to the f16 storage precision, exactly equal for f32 plans' CUDA-core path
    bulk = cuda_forward_bulk(be, m, ids, 32, chunk_tokens=48)
    for b, g in zip(bulk, got):
        assert np.allclose(b, g, rtol=2e-3, atol=2e-3), np.abs(np.asarray(b) - np.asarray(g)).max()


def baseline_case(name, layers, lengths, bucket, seed=7):
    cfg = dict(synthetic.CONFIGS[name]["config"])
    if name == "distilbert":
        cfg["n_layers"] = layers
    else:
        cfg["num_hidden_layers"] = layers
    cfg["vocab_size"] = 512
    if name == "deberta-v3-base":
        pass
    m = Model(cfg, synthetic.CONFIGS[name]["extras"], seed=seed, f16=synthetic.CONFIGS[name]["f16"])
    c = synthetic.CONFIGS[name]
    ids = synthetic.token_ids(name, lengths, seed)
    ids = [np.minimum(x, 511) for x in ids]
    return m, ids


@pytest.mark.parametrize("name,layers,lengths,bucket", [
    ("minilm-l6", 2, [128, 77], 128),
    ("roberta-base", 2, [128, 40], 128),
    ("deberta-v3-base", 1, [512, 300], 512),
    ("modernbert-base", 3, [45, 200, 8, 512], 512),
    ("mminilm-l12-xlmr", 2, [142, 36, 300], 512),
])
def test_baseline_configs_full_width(name, layers, lengths, bucket, backend_factory):
    m, ids = baseline_case(name, layers, lengths, bucket)
    be = backend_factory(m)
    want = oracle_forward(m, ids, bucket, threads=8)
    got = cuda_forward_plan(be, m, ids, bucket)
    (assert_f16 if m.f16 else assert_f32)(got, want)
    bulk = cuda_forward_bulk(be, m, ids, bucket, chunk_tokens=max(bucket, 600))
    assert np.allclose(bulk, got, rtol=2e-3, atol=2e-3), np.abs(bulk - got).max()


def test_batch_plan_matches_single_calls(backend_factory):
    """A batch plan (B = 4 at a 64-row stride, src/encoder.ts:407-448) gives each row's B = 1 output."""
    from kleinhirn_b200.encoder import Encoder
    case = GOLDEN["cases"][1]
    m = Model(case["config"], case["extras"], seed=case["seed"], f16=True)
    be = backend_factory(m)
    enc = Encoder(be, m.spec, m.head, m.word_table, buckets=(32, 64), f16=True)
    rng = np.random.default_rng(3)
    id_lists = [list(rng.integers(3, 96, n)) for n in (5, 17, 31, 9, 60, 2)]
    single = np.stack([enc.run_ids(x) for x in id_lists])
    batched = np.stack(enc.run_ids_batch(id_lists))
    ragged = enc.run_ragged(id_lists)
    assert np.allclose(batched, single, atol=1e-3), np.abs(batched - single).max()
    assert np.allclose(ragged, single, atol=2e-3), np.abs(ragged - single).max()


def words_row_checksum(row: np.ndarray, row_id: int, salt: int) -> int:
    """The row checksum of words.bin (murmur3_32 body over the row's u32 words, seeded with the salt
    and the row id; src/words-format.ts:19-33), so the test file has the reference's layout."""
    M = 0xFFFFFFFF

    def rotl(x, r):
        return ((x << r) | (x >> (32 - r))) & M
    h = (salt ^ ((row_id + 1) * 0x9E3779B1 & M)) & M
    for k in np.frombuffer(row.tobytes(), dtype="<u4"):
        k = int(k) * 0xCC9E2D51 & M
        k = rotl(k, 15)
        k = k * 0x1B873593 & M
        h ^= k
        h = rotl(h, 13)
        h = (h * 5 + 0xE6546B64) & M
    h ^= row.size
    h ^= h >> 16
    h = h * 0x85EBCA6B & M
    h ^= h >> 13
    h = h * 0xC2B2AE35 & M
    h ^= h >> 16
    return h


def test_bulk_ids_gathered_on_device(backend_factory):
    """kh_bulk_upload_ids with the word table on the device gives the bits of kh_bulk_upload with
    host-gathered word rows; an id outside the table is reported by the next read."""
    from kleinhirn_b200.backend import KhError
    from kleinhirn_b200.encoder import packed_inputs
    from kleinhirn_b200.plan import build_plan
    m, ids = baseline_case("mminilm-l12-xlmr", 2, [142, 36, 300, 7], 512)
    be = backend_factory(m)
    be.add_tensor("embeddings.word.weight", m.word_table)
    plan = build_plan(m.spec, m.head, 512, 1, 0, m.f16)
    r = be.runner(plan)
    emb, types, lens = packed_inputs(m.spec, m.word_table, [np.asarray(x) for x in ids])
    flat = np.concatenate([np.asarray(x, dtype=np.int32) for x in ids])
    tt = types if "typeIds" in plan["inputs"] else None
    bulk = be.bulk(r, int(lens.sum()), len(lens), 600)
    want = bulk.run_batch(lens, emb, tt)
    bulk.set_word_table("embeddings.word.weight")
    for _ in range(2):
        bulk.set_lengths(lens)
        bulk.upload_ids(flat, tt)
        bulk.run()
        got = bulk.read()
        assert np.array_equal(got, want)
    # the same table from words.bin bytes: rows of values plus a checksum word (src/words-format.ts)
    table = np.ascontiguousarray(m.word_table)
    vocab, width = table.shape
    row_bytes = width * table.itemsize + 4
    words = np.zeros((vocab, row_bytes), dtype=np.uint8)
    words[:, : width * table.itemsize] = table.view(np.uint8).reshape(vocab, -1)
    words[:, -4:] = np.array([words_row_checksum(words[i, :-4], i, 7) for i in range(vocab)],
                             dtype="<u4").view(np.uint8).reshape(vocab, 4)
    be.add_words("words.bin", words.tobytes(), "f16" if m.f16 else "f32", vocab, width, row_bytes)
    bulk.set_word_table("words.bin")
    bulk.set_lengths(lens)
    bulk.upload_ids(flat, tt)
    bulk.run()
    assert np.array_equal(bulk.read(), want)
    bad = flat.copy()
    bad[5] = m.spec["vocab"]
    bulk.set_lengths(lens)
    bulk.upload_ids(bad, tt)
    bulk.run()
    with pytest.raises(KhError, match="outside the word table"):
        bulk.read()
    bulk.close()
    r.destroy()

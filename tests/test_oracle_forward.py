"""The oracle end to end against the reference's own float64 forward (convert/k28_forward.py),
through the committed golden file tests/golden/forward_golden.json (made by
tests/golden/make_golden.py), for every family: BERT, RoBERTa, XLM-R, DistilBERT, DeBERTa-v3,
ModernBERT."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from harness import Model, oracle_forward

GOLDEN = json.loads((Path(__file__).parent / "golden" / "forward_golden.json").read_text())


def digest(tensors):
    h = hashlib.sha256()
    for k in sorted(tensors):
        h.update(k.encode())
        h.update(np.ascontiguousarray(tensors[k], dtype=np.float32).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
def test_oracle_matches_reference_f64_forward(case):
    m = Model(case["config"], case["extras"], seed=case["seed"])
    assert digest(m.weights) == case["weights_sha256"], "weight generator changed: regenerate the golden file"
    ids = [it["ids"] for it in case["items"]]
    got = oracle_forward(m, ids, 32)
    for g, it in zip(got, case["items"]):
        want = np.array(it["want"])
        scale = max(1.0, np.abs(want).max())
        assert np.abs(g - want).max() <= 2e-5 * scale, (case["name"], np.abs(g - want).max())
        cos = g @ want / (np.linalg.norm(g) * np.linalg.norm(want))
        assert cos >= 0.99999


def test_oracle_threads_match_serial():
    case = GOLDEN["cases"][0]
    m = Model(case["config"], case["extras"], seed=case["seed"])
    ids = [it["ids"] for it in case["items"]]
    a = oracle_forward(m, ids, 32, threads=1)
    b = oracle_forward(m, ids, 32, threads=3)
    assert np.array_equal(a, b)

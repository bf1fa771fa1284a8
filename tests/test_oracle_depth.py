"""The oracle (the restated WASM executor, f32) at the full depth, width and vocabulary of the five
benchmark configurations, against the reference's float64 executable specification
(tests/golden/depth_golden.json, from convert/k28_forward.py:148-283 on the same weights and ids).
This pins the checker the GPU tests and the bench's parity block use at the depth they run at."""
import hashlib
import json
import os
from pathlib import Path

import numpy as np
import pytest

from harness import Model, cosine_rows, oracle_forward
from kleinhirn_b200 import synthetic

GOLDEN = json.loads((Path(__file__).parent / "golden" / "depth_golden.json").read_text())
# f32 arithmetic of the oracle against float64 on the same values: measured at most 1.4e-6
ORACLE_ABS = 1e-5


def weights_digest(tensors):
    h = hashlib.sha256()
    for k in sorted(tensors):
        h.update(k.encode())
        h.update(np.ascontiguousarray(tensors[k]).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
def test_oracle_at_full_depth(case):
    c = synthetic.CONFIGS[case["name"]]
    m = Model(c["config"], c["extras"], seed=GOLDEN["seed"], f16=case["f16"])
    assert weights_digest(m.weights) == case["weights_sha256"], "weight generator changed"
    ids = [np.asarray(it["ids"]) for it in case["items"]]
    want = np.array([it["want"] for it in case["items"]], dtype=np.float64)
    bucket = 128 if max(len(x) for x in ids) <= 128 else 512
    got = np.asarray(oracle_forward(m, ids, bucket, threads=min(os.cpu_count() or 1, 8)), dtype=np.float64)
    assert np.abs(got - want).max() <= ORACLE_ABS
    if want.shape[1] > 1:
        assert cosine_rows(got, want).min() >= 0.99999

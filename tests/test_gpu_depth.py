"""Parity of the five benchmark configurations at full depth, width and vocabulary, through the C
ABI, against the reference's own numpy specifications (tests/golden/depth_golden.json, written by
tests/golden/make_depth_golden.py from convert/k28_forward.py and convert/k28_f16_sim.py) and
against the oracle (the restated WASM executor, f32) run here on the same weights and ids.

Acceptance (with the reference's own f16 gate):
- f32 plans (config 1): cosine >= 0.9999 against the float64 specification and the oracle;
- f16 plans: cosine >= 0.999, and every output within 3 * delta_sim of the float64
  specification, where delta_sim is the largest deviation of the reference's own f16 simulation
  of its engine on the same weights and ids (the rule of convert/k28_f16_sim.py:9-11); against
  the oracle the same bound applies (the oracle's f32 arithmetic is within 1e-5 of float64);
- classifiers: the same argmax as the float64 specification wherever its top two logits are
  further apart than twice the tolerance;
- the ragged bulk path (the bench's path) gives the B = 1 plan results within 2e-3.
"""
import hashlib
import json
import os
from pathlib import Path

import numpy as np
import pytest

from harness import Model, cosine_rows, cuda_forward_bulk, cuda_forward_plan, oracle_forward
from kleinhirn_b200 import synthetic

pytestmark = pytest.mark.gpu

GOLDEN = json.loads((Path(__file__).parent / "golden" / "depth_golden.json").read_text())
CASES = {c["name"]: c for c in GOLDEN["cases"]}
ORACLE_F32_SLACK = 1e-5


def weights_digest(tensors):
    h = hashlib.sha256()
    for k in sorted(tensors):
        h.update(k.encode())
        h.update(np.ascontiguousarray(tensors[k]).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("name", list(CASES))
def test_full_depth_against_reference_spec(name):
    from kleinhirn_b200.backend import CudaBackend
    case = CASES[name]
    c = synthetic.CONFIGS[name]
    m = Model(c["config"], c["extras"], seed=GOLDEN["seed"], f16=case["f16"])
    assert m.spec["layers"] == case["layers"] and m.spec["vocab"] == case["vocab"]
    assert weights_digest(m.weights) == case["weights_sha256"], "weight generator changed"
    ids = [np.asarray(it["ids"]) for it in case["items"]]
    want = np.array([it["want"] for it in case["items"]], dtype=np.float64)
    bucket = 128 if max(len(x) for x in ids) <= 128 else 512
    oracle = np.asarray(oracle_forward(m, ids, bucket, threads=min(os.cpu_count() or 1, 16)), dtype=np.float64)
    be = CudaBackend(m.weights)
    try:
        got = np.asarray(cuda_forward_plan(be, m, ids, bucket), dtype=np.float64)
        bulk = np.asarray(cuda_forward_bulk(be, m, ids, bucket, chunk_tokens=4096), dtype=np.float64)
    finally:
        be.dispose()
    if case["f16"]:
        tol = 3.0 * case["delta_sim"]
        cos_min = 0.999
    else:
        tol = None
        cos_min = 0.9999
    for ref_name, ref in (("float64 spec", want), ("oracle", oracle)):
        if got.shape[1] > 1:
            cos = cosine_rows(got, ref)
            assert cos.min() >= cos_min, f"{ref_name}: cosine {cos.min()}"
        else:  # one logit per sequence: the cosine of the logit vector
            g, r = got.ravel(), ref.ravel()
            assert g @ r / (np.linalg.norm(g) * np.linalg.norm(r)) >= cos_min
        if tol is not None:
            slack = 0.0 if ref is want else ORACLE_F32_SLACK
            err = np.abs(got - ref).max()
            assert err <= tol + slack, f"{ref_name}: max |diff| {err:.3e} above 3 * delta_sim = {tol:.3e}"
    if m.head["type"] == "classify" and want.shape[1] > 1:
        top2 = np.sort(want, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 2 * (tol or 1e-4)
        assert np.array_equal(np.argmax(got, 1)[clear], np.argmax(want, 1)[clear])
    assert np.allclose(bulk, got, rtol=2e-3, atol=2e-3), np.abs(bulk - got).max()

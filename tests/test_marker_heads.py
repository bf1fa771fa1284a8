"""GLiNER2 and Julia marker heads (src/plan/build.ts:358-430): the marker gather, the head
matmuls, masklogits, and Julia's type rows and head layers.

The golden logits (tests/golden/marker_golden.json) come from the reference's float64
executable specifications (convert/manifest_forward.py, convert/julia_manifest_forward.py) on
tiny random-init models. The oracle (the restated WASM executor, f32) must reproduce them; the
CUDA backend must match the oracle, B = 1 per text and as one batch plan with per-sequence type
rows, through kh_upload_markers."""
import json
from pathlib import Path

import numpy as np
import pytest

from kleinhirn_b200.plan import build_plan
from kleinhirn_b200.spec import spec_from_gliner_manifest, spec_from_julia_manifest
from kleinhirn_b200.synthetic import random_weights, to_f16
from oracle import host

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "marker_golden.json").read_text())
CASES = {c["name"]: c for c in GOLDEN["cases"]}
FILL = -1e4


def model(case: dict):
    if case["kind"] == "gliner2":
        spec, head = spec_from_gliner_manifest(case["encoder"], case["head"], case["markers"])
    else:
        spec, head = spec_from_julia_manifest(case["encoder"])
    return spec, head, random_weights(spec, head, seed=case["seed"])


def packed(items: list[dict], K: int) -> np.ndarray:
    """RunInput.packedMarkers: per sequence [K indices | K mask words (f32 bits) | K groups]."""
    blocks = []
    for it in items:
        blocks += [np.asarray(it["markers"], np.uint32), np.asarray(it["mask"], np.float32).view(np.uint32),
                   np.asarray(it["groups"], np.uint32)]
    return np.concatenate(blocks)


def inputs(items: list[dict], table: np.ndarray, L: int, dtype):
    """Word rows and prefix masks of a batch of texts at an L-row stride."""
    emb = np.zeros((len(items) * L, table.shape[1]), dtype=dtype)
    mask = np.zeros(len(items) * L, dtype=np.float32)
    for b, it in enumerate(items):
        n = len(it["ids"])
        emb[b * L: b * L + n] = table[np.asarray(it["ids"])]
        mask[b * L: b * L + n] = 1.0
    return emb, mask


def qtypes(items):
    return [it.get("qtype", 0) for it in items]


def oracle_logits(case: dict, items: list[dict], batch: int = 1) -> np.ndarray:
    spec, head, w = model(case)
    L, K = case["length"], case["markers"]
    plan = build_plan(spec, head, L, batch, K, False)
    rt = host.Runtime(threads=2)
    try:
        host.load_weights(rt, w, [plan])
        p = rt.plan(plan)
        outs = []
        groups = [items[i:i + batch] for i in range(0, len(items), batch)]
        for g in groups:
            emb, mask = inputs(g, w["embeddings.word.weight"], L, np.float32)
            p.upload(emb, mask, None, packed(g, K), qtypes(g) if batch > 1 else qtypes(g)[0])
            p.run(len(g[0]["ids"]) if batch == 1 else L * batch)
            outs.append(p.read_output()[: K * len(g)])
        return np.concatenate(outs)
    finally:
        rt.close()


def check_logits(got: np.ndarray, want: np.ndarray, atol: float, rtol: float, what: str):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    off = want == FILL
    assert np.all(got[off] == FILL), f"{what}: masked markers must read exactly -1e4"
    err = np.abs(got[~off] - want[~off])
    tol = atol + rtol * np.abs(want[~off])
    assert np.all(err <= tol), f"{what}: worst {err.max():.3g} (tolerance {tol[np.argmax(err - tol)]:.3g})"


@pytest.mark.parametrize("name", sorted(CASES))
def test_weights_are_the_recorded_ones(name):
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    from make_golden import weights_digest
    _, _, w = model(CASES[name])
    assert weights_digest(w) == CASES[name]["weights_sha256"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_the_reference_spec(name):
    case = CASES[name]
    want = np.concatenate([it["logits"] for it in case["items"]])
    # f32 oracle against the f64 specification
    check_logits(oracle_logits(case, case["items"]), want, 2e-5, 1e-3, f"{name} oracle")


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_batch_plan_equals_single_calls(name):
    case = CASES[name]
    single = oracle_logits(case, case["items"])
    batch = oracle_logits(case, case["items"], batch=len(case["items"]))
    check_logits(batch, single, 1e-6, 1e-5, f"{name} oracle batch")


def cuda_logits(backend, case: dict, items: list[dict], f16: bool, batch: int = 1) -> np.ndarray:
    spec, head, w = model(case)
    L, K = case["length"], case["markers"]
    plan = build_plan(spec, head, L, batch, K, f16)
    r = backend.runner(plan)
    table = to_f16({"t": w["embeddings.word.weight"]})["t"] if f16 else w["embeddings.word.weight"]
    outs = []
    try:
        for i in range(0, len(items), batch):
            g = items[i:i + batch]
            emb, mask = inputs(g, table, L, np.float16 if f16 else np.float32)
            r.upload(emb, mask, None, packed(g, K), qtypes(g))
            r.run(len(g[0]["ids"]) if batch == 1 else L * batch)
            outs.append(r.read_output()[: K * len(g)])
    finally:
        r.destroy()
    return np.concatenate(outs)


@pytest.fixture(scope="module")
def backends():
    from kleinhirn_b200.backend import CudaBackend
    out = {}
    for name, case in CASES.items():
        spec, head, w = model(case)
        for f16 in (False, True):
            out[(name, f16)] = CudaBackend(to_f16(w) if f16 else w)
    yield out
    for b in out.values():
        b.dispose()


@pytest.mark.gpu
@pytest.mark.parametrize("f16", [False, True], ids=["f32", "f16"])
@pytest.mark.parametrize("name", sorted(CASES))
def test_cuda_marker_head_matches_oracle(backends, name, f16):
    case = CASES[name]
    want = oracle_logits(case, case["items"])
    got = cuda_logits(backends[(name, f16)], case, case["items"], f16)
    scale = float(np.abs(want[want != FILL]).max())
    if f16:  # f16 storage: 2e-2 of the logit scale
        check_logits(got, want, 2e-2 * scale, 0.0, f"{name} f16")
    else:
        check_logits(got, want, 1e-4 * scale, 1e-4, f"{name} f32")
    golden = np.concatenate([it["logits"] for it in case["items"]])
    check_logits(got, golden, (2e-2 if f16 else 1e-4) * scale, 1e-4, f"{name} vs reference spec")


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_cuda_batch_plan_with_type_rows(backends, name):
    """One batch plan of all texts (each its own qtype for Julia) gives the B = 1 results."""
    case = CASES[name]
    single = cuda_logits(backends[(name, False)], case, case["items"], False)
    batch = cuda_logits(backends[(name, False)], case, case["items"], False, batch=len(case["items"]))
    scale = float(np.abs(single[single != FILL]).max())
    check_logits(batch, single, 1e-4 * scale, 1e-4, f"{name} batch plan")


@pytest.mark.gpu
def test_upload_markers_checks_its_arguments(backends):
    from kleinhirn_b200.backend import KhError
    case = CASES["julia-tiny"]
    spec, head, w = model(case)
    L, K = case["length"], case["markers"]
    r = backends[("julia-tiny", False)].runner(build_plan(spec, head, L, 1, K, False))
    try:
        it = case["items"][0]
        emb, mask = inputs([it], w["embeddings.word.weight"], L, np.float32)
        with pytest.raises(KhError, match="packedMarkers"):  # as the reference's upload
            r.upload(emb, mask)
        with pytest.raises(KhError, match="packedMarkers"):  # the library refuses the run too
            r.run(len(it["ids"]))
        with pytest.raises(KhError, match="qtype 3 outside"):
            r.upload(emb, mask, None, packed([it], K), [3])
        with pytest.raises(KhError, match="words"):
            r.upload(emb, mask, None, np.zeros(3 * K + 1, np.uint32), [0])
    finally:
        r.destroy()

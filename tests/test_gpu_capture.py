"""Layer capture through the C ABI (kh_capture_check / kh_run_capture / kh_read_capture), the
CUDA form of PlanRunner.run(seqLen, true) + readCapture (src/plan/executor.ts:178-186, :232,
:267-281, :418-424): one forward over the full bucket that runs each segment's captureOps and
copies the segment's capture buffers into their slots. Each slot must equal the oracle's buffer
after the same segments (a plan cut after that segment, captureOps run in place)."""
import sys
from pathlib import Path

import numpy as np
import pytest

from harness import Model
from kleinhirn_b200.encoder import mask_and_types, word_rows
from kleinhirn_b200.plan import build_plan
from oracle import host

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_golden import CASES  # noqa: E402  (configs of the tiny family members)

pytestmark = pytest.mark.gpu
BY_NAME = {c["name"]: c for c in CASES}


def oracle_slots(m: Model, plan: dict, emb, mask, types) -> dict[int, np.ndarray]:
    """Slot -> the captured buffer's first captureSlotBytes, from the oracle run on the plan cut
    after the capturing segment."""
    L = plan["length"]
    out = {}
    for s, seg in enumerate(plan["segments"]):
        if not seg.get("capture"):
            continue
        cut = dict(plan)
        cut["segments"] = [{**g, "ops": list(g.get("captureOps", [])) + list(g["ops"]), "captureOps": []}
                           for g in plan["segments"][: s + 1]]
        rt = host.Runtime(threads=2)
        try:
            host.load_weights(rt, m.weights32, [cut])
            p = rt.plan(cut)
            p.upload(emb, mask, types)
            p.run(L)  # capture keeps the full bucket
            for c in seg["capture"]:
                v = p.view(c["buffer"])
                out[c["slot"]] = v[: plan["captureSlotBytes"] // 4].copy()
        finally:
            rt.close()
    return out


@pytest.mark.parametrize("name", ["bert-embed-mean", "deberta-v3-classify", "modernbert-embed"])
def test_capture_slots_match_the_oracle(name):
    from kleinhirn_b200.backend import CudaBackend
    case = BY_NAME[name]
    m = Model(case["config"], case["extras"], seed=case["seed"])
    L = 32
    plan = build_plan(m.spec, m.head, L, 1, 0, False)
    ids = np.random.default_rng(5).integers(3, m.spec["vocab"], 21)
    inputs = [{"inputIds": ids.tolist()}]
    mask, types = mask_and_types(m.spec, inputs, L)
    emb = word_rows(m.weights32["embeddings.word.weight"], inputs, L)
    want = oracle_slots(m, plan, emb, mask, types)
    be = CudaBackend(m.weights)
    try:
        r = be.runner(plan)
        r.upload(emb, mask, types)
        r.run(len(ids), capture=True)
        got = r.read_capture().reshape(plan["captureSlots"], -1)
        out_capture = r.read_output()
        r.run(len(ids))  # a plain run afterwards gives the same output
        assert np.allclose(r.read_output(), out_capture, rtol=1e-5, atol=1e-6)
        r.destroy()
    finally:
        be.dispose()
    assert sorted(want) == list(range(plan["captureSlots"]))
    for slot, w in want.items():
        scale = float(np.abs(w).max())
        err = float(np.abs(got[slot] - w).max())
        assert err <= 1e-4 * scale, f"{name} slot {slot}: worst {err:.3g} of scale {scale:.3g}"


def test_capture_is_refused_as_the_reference_refuses():
    from kleinhirn_b200.backend import CudaBackend, KhError
    case = BY_NAME["bert-embed-mean"]
    m = Model(case["config"], case["extras"], seed=case["seed"], f16=True)
    be = CudaBackend(m.weights)
    try:
        r16 = be.runner(build_plan(m.spec, m.head, 32, 1, 0, True))
        with pytest.raises(KhError, match="capture needs an f32 plan"):
            r16.assert_capturable()
        r16.destroy()
        r2 = be.runner(build_plan(m.spec, m.head, 32, 2, 0, False))
        with pytest.raises(KhError, match="capture needs a plan of batch 1, this one has 2"):
            r2.run(64, capture=True)
        r2.destroy()
    finally:
        be.dispose()

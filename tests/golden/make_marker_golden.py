"""Generates tests/golden/marker_golden.json: logits of tiny random-init GLiNER2 and Julia models,
computed by the reference's own float64 executable specifications imported from the reference
checkout:

- GLiNER2 (DeBERTa-v3 encoder + marker head): ``convert/manifest_forward.py`` ``forward``
  (convert/manifest_forward.py:88-155): states at the marker rows, ReLU(fc1), fc2, / temperature,
  -1e4 where the marker mask is off;
- Julia (ModernBERT encoder + typed head): ``convert/julia_manifest_forward.py``
  ``julia_forward`` (convert/julia_manifest_forward.py:119-171), whose docstring states the
  -1e4 fill on invalid markers; the function returns raw scores, so the fill is applied here.

Both specs fix their constants: LayerNorm eps 1e-7 (GLiNER2) and 1e-5 (Julia), RoPE over a head
dimension of 64 (Julia), so the tiny models keep those. Run in the build container, where the
reference exists:

    python tests/golden/make_marker_golden.py <path to the reference checkout>

The weights are regenerated from the recorded seeds by kleinhirn_b200.synthetic.random_weights;
the file records their sha256 so a change of the generator fails the tests. The tests read the
JSON only; they never import the reference.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from kleinhirn_b200.spec import spec_from_gliner_manifest, spec_from_julia_manifest  # noqa: E402
from kleinhirn_b200.synthetic import random_weights  # noqa: E402

sys.path.insert(0, str(Path(__file__).resolve().parent))
from make_golden import weights_digest  # noqa: E402

OUT = Path(__file__).resolve().parent / "marker_golden.json"

# GLiNER2: manifest `encoder` fields (src/plan/spec.ts:187-196) plus the head's temperature.
GLINER = {"name": "gliner2-tiny", "seed": 31, "length": 48, "markers": 6,
          "encoder": {"hiddenSize": 128, "layers": 2, "heads": 2, "intermediateSize": 192, "positionBuckets": 16,
                      "maxRelativePositions": 64, "layerNormEps": 1e-7, "vocabSize": 96},
          "head": {"temperature": 0.7, "hiddenSize": 96},
          "lengths": [48, 19, 33]}
# Julia: src/plan/spec.ts:198-212 fields; three layers so layer 0 is global and 1, 2 are windowed.
JULIA = {"name": "julia-tiny", "seed": 32, "length": 40,
         "encoder": {"layers": 3, "hiddenSize": 128, "heads": 2, "intermediate": 96, "normEps": 1e-5,
                     "ropeTheta": 160000.0, "localAttention": 8, "globalEvery": 3, "headLayers": 2, "headFfn": 160,
                     "options": 5, "vocab": 96},
         "lengths": [40, 23, 12], "qtypes": [2, 0, 1]}


def _markers(rng, n: int, k: int) -> tuple[list[int], list[float], list[int]]:
    idx = sorted(rng.choice(n, size=min(k, n), replace=False).tolist())
    idx += [0] * (k - len(idx))
    mask = [1.0] * k
    for j in rng.choice(k, size=2, replace=False):  # two markers off: their logits are the fill
        mask[int(j)] = 0.0
    groups = rng.integers(0, 3, k).tolist()
    return idx, mask, groups


def main(ref: Path) -> None:
    sys.path.insert(0, str(ref / "convert"))
    import julia_manifest_forward as jf  # the reference's executable specifications
    import manifest_forward as mf

    rng = np.random.default_rng(2025)
    out = {"source": "convert/manifest_forward.py forward, convert/julia_manifest_forward.py julia_forward; float64",
           "cases": []}

    spec, head = spec_from_gliner_manifest(GLINER["encoder"], GLINER["head"], GLINER["markers"])
    w = random_weights(spec, head, seed=GLINER["seed"])
    T = {k: v.astype(np.float64) for k, v in w.items()}
    enc = {"heads": spec["heads"], "hiddenSize": spec["hidden"], "layers": spec["layers"],
           "positionBuckets": GLINER["encoder"]["positionBuckets"],
           "maxRelativePositions": GLINER["encoder"]["maxRelativePositions"],
           "temperature": GLINER["head"]["temperature"]}
    items = []
    for n in GLINER["lengths"]:
        ids = rng.integers(1, spec["vocab"], n)
        idx, mask, groups = _markers(rng, n, GLINER["markers"])
        logits = mf.forward(T, enc, ids, np.ones(n), np.asarray(idx), np.asarray(mask))
        items.append({"ids": ids.tolist(), "markers": idx, "mask": mask, "groups": groups,
                      "logits": [float(v) for v in logits]})
    out["cases"].append({**{k: GLINER[k] for k in ("name", "seed", "length", "markers", "encoder", "head")},
                         "kind": "gliner2", "weights_sha256": weights_digest(w), "items": items})

    spec, head = spec_from_julia_manifest(JULIA["encoder"])
    w = random_weights(spec, head, seed=JULIA["seed"])
    T = {k: v.astype(np.float64) for k, v in w.items()}
    cfg = {"layers": spec["layers"], "heads": spec["heads"], "localAttention": JULIA["encoder"]["localAttention"],
           "globalEvery": JULIA["encoder"]["globalEvery"], "ropeTheta": JULIA["encoder"]["ropeTheta"],
           "intermediate": spec["intermediate"], "headLayers": JULIA["encoder"]["headLayers"]}
    K = JULIA["encoder"]["options"]
    items = []
    for n, q in zip(JULIA["lengths"], JULIA["qtypes"]):
        ids = rng.integers(1, spec["vocab"], n)
        idx, mask, groups = _markers(rng, n, K)
        s = jf.julia_forward(T, cfg, ids.tolist(), np.ones(n), idx, q, dtype=np.float64)
        logits = np.where(np.asarray(mask) > 0.5, s, -1e4)
        items.append({"ids": ids.tolist(), "markers": idx, "mask": mask, "groups": groups, "qtype": q,
                      "logits": [float(v) for v in logits]})
    out["cases"].append({**{k: JULIA[k] for k in ("name", "seed", "length", "encoder")}, "markers": K,
                         "kind": "julia", "weights_sha256": weights_digest(w), "items": items})
    OUT.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_marker_golden.py <path to the reference checkout>")
    main(Path(sys.argv[1]))

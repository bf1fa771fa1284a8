"""The plan builder (kleinhirn_b200/plan.py) against the reference's frozen dispatch lists.

The reference records, through a mock GPU, every write, copy, pipeline (override constants),
bind group and dispatch its WebGPU executor issues for GLiNER2 (DeBERTa-v3 small and base) and
Julia (ModernBERT) plans (tests/plan_trace.test.ts, tests/helpers/plan-trace.ts). The fixture
tests/golden/plan_traces.json.gz holds the plain forward modes of that file. Here the plans
come from the Python builder and the executor's encoding is replayed
(src/plan/executor.ts:202-212 op choice and dispatch sizes, :236-246 type rows, :366-388
uploads, :259-281 one pass and the output copy); buffers are named by first use, as the
recorder does, so the event lists must be equal. Buffer sizes must be equal too, and the
build-time contents (relidx, cossin, zero) must have the recorded sha256: that pins the DeBERTa
relative-position buckets and the RoPE tables bit for bit. Pipelines are recorded as a hash of
the shader source; each (kernel, precision) must map to one hash throughout.
"""
import gzip
import hashlib
import json
import math
import re
from pathlib import Path

from kleinhirn_b200.plan import build_plan
from kleinhirn_b200.spec import spec_from_gliner_manifest, spec_from_julia_manifest

FIXTURE = Path(__file__).resolve().parent / "golden" / "plan_traces.json.gz"

# tests/helpers/plan-trace.ts:24-45
GLINER_SPECS = {
    "small": {"hiddenSize": 384, "layers": 12, "heads": 6, "intermediateSize": 1536, "positionBuckets": 256,
              "maxRelativePositions": 512, "layerNormEps": 1e-7},
    "base": {"hiddenSize": 768, "layers": 12, "heads": 12, "intermediateSize": 3072, "positionBuckets": 256,
             "maxRelativePositions": 512, "layerNormEps": 1e-7},
}
GLINER_HEAD_HIDDEN = {"small": 768, "base": 1536}
JULIA_SPEC = {"layers": 22, "hiddenSize": 384, "heads": 6, "intermediate": 1152, "normEps": 1e-5,
              "ropeTheta": 160000, "localAttention": 64, "globalEvery": 3, "headLayers": 2, "headFfn": 1536,
              "options": 20}


def js_number(x) -> str:
    """Number.prototype.toString: the shortest round-trip digits, positional for decimal
    exponents in (-7, 21), exponential otherwise."""
    x = float(x)
    if x == 0:
        return "0"
    sign = "-" if x < 0 else ""
    mant, _, exp = repr(abs(x)).partition("e")
    ip, _, fp = mant.partition(".")
    if fp == "0":
        fp = ""
    alld = ip + fp
    lead = len(alld) - len(alld.lstrip("0"))
    digits = alld.lstrip("0").rstrip("0")
    n = len(ip) + (int(exp) if exp else 0) - lead  # value = 0.digits x 10^n
    k = len(digits)
    if k <= n <= 21:
        s = digits + "0" * (n - k)
    elif 0 < n <= 21:
        s = digits[:n] + "." + digits[n:]
    elif -6 < n <= 0:
        s = "0." + "0" * (-n) + digits
    else:
        e = n - 1
        s = digits[0] + ("." + digits[1:] if k > 1 else "") + "e" + ("+" if e >= 0 else "-") + str(abs(e))
    return sign + s


def test_js_number():
    assert [js_number(v) for v in (1e-5, 1e-7, 0.125, 160000, 1.0, 384, 1e21, 123.5, 0.000123)] == \
        ["0.00001", "1e-7", "0.125", "160000", "1", "384", "1e+21", "123.5", "0.000123"]


def dim(d, rows: int) -> int:
    """src/plan/executor.ts:202-204."""
    return {"rows": rows, "rows8": math.ceil(rows / 8), "rows16": math.ceil(rows / 16),
            "rows32": math.ceil(rows / 32)}.get(d, d) if isinstance(d, str) else d


def replay(plan: dict, rows: int, qtypes: list[int]) -> list[list]:
    """The executor's events for upload + one forward over ``rows`` rows + the output copy,
    with plan buffer ids (kernels stand in for the pipeline hashes)."""
    size = {d["id"]: d["bytes"] for d in plan["buffers"]}
    ev: list[list] = []
    inp = plan["inputs"]
    ev.append(["write", inp["embeddings"], 0, size[inp["embeddings"]]])
    ev.append(["write", inp["mask"], 0, size[inp["mask"]]])
    if "kinfo" in size:
        ev.append(["write", "kinfo", 0, 8 * plan["batch"]])
    if inp.get("markers"):
        ev.append(["write", inp["markers"], 0, size[inp["markers"]]])
    if inp.get("typeIds"):
        ev.append(["write", inp["typeIds"], 0, size[inp["typeIds"]]])
    rs = plan.get("rowSelect")
    if rs:
        for b in range(plan["batch"]):
            q = qtypes[b] if b < len(qtypes) else 0
            ev.append(["copy", rs["table"], q * rs["rowBytes"], rs["dst"], b * rs["rowBytes"], rs["rowBytes"]])
    ev.append(["begin"])
    for seg in plan["segments"]:
        for op in seg["ops"]:
            o = next((a for a in op.get("alts", []) if rows <= a["maxRows"]), op)
            consts = ",".join(f"{k}={js_number(op['constants'][k])}" for k in sorted(op["constants"]))
            ev.append(["pipe", (o["kernel"], plan["f16"]), consts])
            ev.append(["bind", 0, [[i, b] for i, b in enumerate(op["bind"])]])
            ev.append(["dispatch", dim(o["dispatch"][0], rows), dim(o["dispatch"][1], rows)])
    ev.append(["end"])
    ev.append(["copy", plan["output"]["buffer"], 0, "#staging", 0, plan["output"]["bytes"]])
    return ev


def canonical(ev: list[list], pipes: dict) -> tuple[list[str], dict[str, str]]:
    """Names buffers b0, b1, ... by first use (weights keep their names) and pipelines by the
    recorded hash of their kernel."""
    names: dict[str, str] = {}

    def ref(b: str) -> str:
        if b.startswith("w:"):
            return b
        if b not in names:
            names[b] = f"b{len(names)}"
        return names[b]

    out = []
    for e in ev:
        if e[0] == "write":
            out.append(json.dumps(["write", ref(e[1]), e[2], e[3]], separators=(",", ":")))
        elif e[0] == "copy":
            out.append(json.dumps(["copy", ref(e[1]), e[2], ref(e[3]), e[4], e[5]], separators=(",", ":")))
        elif e[0] == "pipe":
            out.append(json.dumps(["pipe", f"{pipes.get(e[1], '?')}|{e[2]}"], separators=(",", ":")))
        elif e[0] == "bind":
            out.append(json.dumps(["bind", 0, [[i, ref(b)] for i, b in e[2]]], separators=(",", ":")))
        else:
            out.append(json.dumps(e, separators=(",", ":")))
    return out, names


def _frozen() -> dict:
    return json.loads(gzip.decompress(FIXTURE.read_bytes()))


def _build(trace_id: str):
    m = re.fullmatch(r"(small|base|julia-1)-(f16|f32)-B(\d+)-L(\d+)K(\d+)-(normal|normal100)", trace_id)
    shape, prec, batch, length, markers, mode = m.groups()
    batch, length, markers = int(batch), int(length), int(markers)
    if shape == "julia-1":
        spec, head = spec_from_julia_manifest(JULIA_SPEC)
        qtypes = [0] if batch == 1 else [0, 1, 2, 0]
    else:
        spec, head = spec_from_gliner_manifest(GLINER_SPECS[shape], {"temperature": 1.0,
                                                                     "hiddenSize": GLINER_HEAD_HIDDEN[shape]})
        qtypes = []
    plan = build_plan(spec, head, length, batch, markers, prec == "f16")
    rows = length * batch if mode == "normal" else 100 * batch
    return plan, rows, qtypes


TRACE_IDS = sorted(_frozen()["traces"]) if FIXTURE.exists() else []


def test_fixture_covers_the_shapes():
    assert len(TRACE_IDS) == 56
    assert {t.split("-")[0] for t in TRACE_IDS} == {"small", "base", "julia"}


def test_plans_replay_the_frozen_dispatch_lists():
    frozen = _frozen()["traces"]
    pipes: dict = {}
    # learn the hash of each (kernel, precision) from its first appearance, then hold it fixed
    bad = []
    for tid in TRACE_IDS:
        plan, rows, qtypes = _build(tid)
        mine = replay(plan, rows, qtypes)
        want = frozen[tid]["events"]
        if len(mine) != len(want):
            bad.append(f"{tid}: {len(mine)} events, recorded {len(want)}")
            continue
        for e, w in zip(mine, want):
            if e[0] == "pipe":
                h = json.loads(w)[1].split("|")[0]
                known = pipes.setdefault(e[1], h)
                assert known == h, f"{tid}: kernel {e[1]} under two shader hashes"
        # (a kernel whose source has no precision switch keeps one hash in f16 and f32 plans)
        owner: dict[str, str] = {}
        for (kern, _), h in pipes.items():
            assert owner.setdefault(h, kern) == kern, f"kernels {kern} and {owner[h]} under one shader hash"
        got, names = canonical(mine, pipes)
        diff = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
        if diff is not None:
            bad.append(f"{tid}: event {diff}: {got[diff]} != {want[diff]}")
            continue
        # buffer sizes and build-time contents
        size = {d["id"]: d["bytes"] for d in plan["buffers"]}
        size["#staging"] = plan["output"]["bytes"]
        init = {d["id"]: d.get("init") for d in plan["buffers"]}
        for bid, bn in names.items():
            rec = frozen[tid]["buffers"][bn]
            if rec["size"] != size[bid]:
                bad.append(f"{tid}: buffer {bid} has {size[bid]} B, recorded {rec['size']}")
            blob = init.get(bid)
            if ("init" in rec) != (blob is not None):
                bad.append(f"{tid}: buffer {bid} init {'missing' if blob is None else 'unexpected'}")
            elif blob is not None and hashlib.sha256(bytes(blob)).hexdigest() != rec["init"]:
                bad.append(f"{tid}: buffer {bid} contents differ from the recorded sha256")
    assert not bad, f"{len(bad)} of {len(TRACE_IDS)} differ:\n" + "\n".join(bad[:8])

"""Plan builder: ModelSpec + HeadSpec -> Plan (the execution plan the CUDA backend runs).

Host-side restatement of ``src/plan/build.ts`` and ``src/plan/layers.ts``. The Plan is the
reference's IR (``src/plan/ir.ts:41-60``): buffers with byte sizes and optional ``init``
blobs, segments of ops (kernel name, override constants, bindings, dispatch), inputs and
output. The TypeScript engine hands exactly this structure to a backend; the CUDA backend
receives it as JSON (``plan_to_json``), ``init`` blobs base64-encoded.

Every constant that reaches a kernel is computed with the expression the reference uses, so
the JSON matches what ``buildPlan`` produces for the same spec.
"""
from __future__ import annotations

import base64
import json
import math
from typing import Any

import numpy as np

from .spec import tensor_names_for

ACT = {"relu": 1, "gelu": 2, "tanh": 3, "silu": 4}
MAX_WORKGROUPS = 65535
SCORES_MAX_BYTES = 134217728


def act_code(act: str) -> int:
    """src/plan/build.ts:91-96."""
    if act not in ACT:
        raise ValueError(f"activation {act} has no kernel yet")
    return ACT[act]


def rel_bucket_index(i: int, j: int, span: int, max_pos: int) -> int:
    """src/plan/build.ts:22-33: DeBERTa log-bucket relative position, f64 arithmetic."""
    rel = i - j
    mid = span >> 1
    a = abs(rel)
    r = rel
    if a > mid:
        log_pos = math.ceil(math.log(a / mid) / math.log((max_pos - 1) / mid) * (mid - 1)) + mid
        r = log_pos * (1 if rel > 0 else -1)
    return min(max(r + span, 0), 2 * span - 1)


def rel_pos_table(length: int, span: int, max_pos: int) -> np.ndarray:
    """src/plan/build.ts:35-45: u32 [L * L], entry i * L + j."""
    t = np.empty(length * length, dtype=np.uint32)
    for i in range(length):
        for j in range(length):
            t[i * length + j] = rel_bucket_index(i, j, span, max_pos)
    return t


def rope_table(length: int, theta: float, head_dim: int) -> np.ndarray:
    """src/plan/build.ts:47-60: f32 [L][cos D | sin D], angles in f64."""
    half = head_dim // 2
    t = np.zeros(length * 2 * head_dim, dtype=np.float32)
    for i in range(length):
        for d in range(half):
            f = i * theta ** (-(2 * d) / head_dim)
            t[i * 2 * head_dim + d] = math.cos(f)
            t[i * 2 * head_dim + head_dim + d] = math.sin(f)
    return t


def writable_bindings(kernel: str, bindings: int) -> list[int]:
    """src/plan/build.ts:64-66."""
    return [0] if kernel in ("add", "rope") else [bindings - 1]


def validate_segments(segments: list[dict], known: set[str]) -> None:
    """src/plan/build.ts:70-87."""
    for seg in segments:
        for op in seg.get("captureOps", []) + seg["ops"]:
            where = f"{seg['prefix']}{op['name']}"
            for i in op["bind"]:
                if not i.startswith("w:") and i not in known:
                    raise ValueError(f"plan op {where}: unknown buffer {i}")
            for wb in writable_bindings(op["kernel"], len(op["bind"])):
                bid = op["bind"][wb]
                if any(k != wb and o == bid for k, o in enumerate(op["bind"])):
                    raise ValueError(f"plan op {where}: writable buffer {bid} is bound twice")


def add_workgroups(rows: int, hidden: int) -> int:
    """src/plan/layers.ts:31-32."""
    return min(math.ceil(rows * hidden / 64), MAX_WORKGROUPS)


def _w(name, zero="zero"):
    return zero if name is None else f"w:{name}"


def _req(name, what):
    if name is None:
        raise ValueError(f"layer tensor {what} missing")
    return f"w:{name}"


def _matmul(name: str, d: dict, n: int, k: int, act: int, bind: list[str]) -> dict:
    """src/plan/layers.ts:36-49."""
    constants = {"M": d["rows"], "N": n, "K": k, "ACT": act}
    if k % 32 == 0:
        return {"name": name, "kernel": "mmtile", "constants": constants, "bind": bind,
                "dispatch": [math.ceil(n / 64), "rows32"],
                "alts": [
                    {"kernel": "mmtile8", "dispatch": [math.ceil(n / 32), "rows8"],
                     "maxRows": 16 * (127 // math.ceil(n / 32))},
                    {"kernel": "mmtile16", "dispatch": [math.ceil(n / 32), "rows16"],
                     "maxRows": 32 * (95 // math.ceil(n / 64))},
                ]}
    return {"name": name, "kernel": "matmul", "constants": constants, "bind": bind,
            "dispatch": [math.ceil(n / 16), "rows16"]}


def _matmul_attention(d: dict) -> bool:
    """src/plan/layers.ts:55-56."""
    return (d["headDim"] % 32 == 0 and d["length"] % 32 == 0
            and d["rows"] * d["heads"] * d["length"] * 4 <= SCORES_MAX_BYTES)


def _relative_attention(d: dict, scale: float, rel: dict, t: dict) -> list[dict]:
    """src/plan/layers.ts:61-80."""
    base = {"L": d["length"], "H": d["heads"], "D": d["headDim"]}
    rel_c = {"H": d["heads"], "D": d["headDim"], "ROWS": d["rows"], "NM": rel["nm"], "MOFF": rel["moff"],
             "L": d["length"]}
    tiles = d["heads"] * math.ceil(rel["nm"] / 64)
    return [
        {"name": "relC", "kernel": "attrel", "constants": {**rel_c, "PART": 0},
         "bind": ["qkv", _req(t.get("posKey"), "posKey"), "kinfo", "relidx", "c2p"], "dispatch": [tiles, "rows32"]},
        {"name": "relP", "kernel": "attrel", "constants": {**rel_c, "PART": 1},
         "bind": ["qkv", _req(t.get("posQuery"), "posQuery"), "kinfo", "relidx", "p2c"],
         "dispatch": [tiles, "rows32"]},
        {"name": "attS", "kernel": "attscore", "constants": {**base, "SCALE": 1 / scale, "ROWS": d["rows"]},
         "bind": ["qkv", "kinfo", "scores"], "dispatch": [d["heads"] * math.ceil(d["length"] / 64), "rows32"]},
        {"name": "attP", "kernel": "attsoftrel",
         "constants": {"L": d["length"], "H": d["heads"], "NM": rel["nm"], "MOFF": rel["moff"],
                       "INVSCALE": 1 / scale},
         "bind": ["mask", "relidx", "c2p", "p2c", "scores"], "dispatch": [d["heads"], "rows"]},
        {"name": "attV", "kernel": "attpv", "constants": {**base, "ROWS": d["rows"]},
         "bind": ["scores", "qkv", "mask", "kinfo", "ctx"], "dispatch": [d["heads"] * (d["headDim"] // 32), "rows32"]},
    ]


def _standard_attention(d: dict, scale: float, window: int) -> list[dict]:
    """src/plan/layers.ts:82-99."""
    base = {"L": d["length"], "H": d["heads"], "D": d["headDim"]}
    if _matmul_attention(d):
        return [
            {"name": "attS", "kernel": "attscore", "constants": {**base, "SCALE": scale, "ROWS": d["rows"]},
             "bind": ["qkv", "kinfo", "scores"], "dispatch": [d["heads"] * math.ceil(d["length"] / 64), "rows32"]},
            {"name": "attP", "kernel": "attsoftmax", "constants": {"L": d["length"], "H": d["heads"], "WINDOW": window},
             "bind": ["mask", "scores"], "dispatch": [d["heads"], "rows"]},
            {"name": "attV", "kernel": "attpv", "constants": {**base, "ROWS": d["rows"]},
             "bind": ["scores", "qkv", "mask", "kinfo", "ctx"],
             "dispatch": [d["heads"] * (d["headDim"] // 32), "rows32"]},
        ]
    constants = {**base, "SCALE": scale, "WINDOW": window}
    if d["headDim"] % 4 == 0 and d["headDim"] <= 64 and d["length"] % 32 == 0:
        return [{"name": "attn", "kernel": "mbflash", "constants": {**constants, "ROWS": d["rows"]},
                 "bind": ["qkv", "mask", "ctx"], "dispatch": [d["heads"], "rows32"]}]
    return [{"name": "attn", "kernel": "mbattention", "constants": constants, "bind": ["qkv", "mask", "ctx"],
             "dispatch": [d["heads"], "rows"]}]


def _layernorm(name: str, d: dict, mode: int, bind: list[str]) -> dict:
    return {"name": name, "kernel": "layernorm", "constants": {"N": d["hidden"], "MODE": mode, "EPS": d["eps"]},
            "bind": bind, "dispatch": ["rows", 1]}


def _add(name: str, d: dict, bind: list[str]) -> dict:
    return {"name": name, "kernel": "add",
            "constants": {"TOTAL": d["rows"] * d["hidden"], "N": d["hidden"], "MODE": 0, "L": d["length"]},
            "bind": bind, "dispatch": [add_workgroups(d["rows"], d["hidden"]), 1]}


def post_norm_layer(d: dict, t: dict, act: int, attn_scale: float, standard: bool, rel: dict | None) -> list[dict]:
    """src/plan/layers.ts:118-149."""
    H, I = d["hidden"], d["intermediate"]
    if standard:
        att = _standard_attention(d, attn_scale, 0)
    elif rel is not None and _matmul_attention(d):
        att = _relative_attention(d, attn_scale, rel, t)
    else:
        att = [{"name": "attn", "kernel": "attention",
                "constants": {"L": d["length"], "H": d["heads"], "D": d["headDim"], "SCALE": attn_scale},
                "bind": ["qkv", _req(t.get("posKey"), "posKey"), _req(t.get("posQuery"), "posQuery"),
                         "relidx", "mask", "ctx"],
                "dispatch": [d["heads"], "rows"]}]
    return [
        _matmul("qkv", d, 3 * H, H, 0, ["x", _req(t.get("qkvW"), "qkvW"), _w(t.get("qkvB")), "qkv"]),
        *att,
        _matmul("attnOut", d, H, H, 0, ["ctx", _req(t.get("attnOutW"), "attnOutW"), _w(t.get("attnOutB")), "attnOut"]),
        _layernorm("lnA", d, 2, ["x", "attnOut", _req(t.get("attnNormW"), "attnNormW"), _w(t.get("attnNormB")),
                                 "mask", "tmp"]),
        _matmul("ffn1", d, I, H, act, ["tmp", _req(t.get("ffnInW"), "ffnInW"), _w(t.get("ffnInB")), "mid"]),
        _matmul("ffn2", d, H, I, 0, ["mid", _req(t.get("ffnOutW"), "ffnOutW"), _w(t.get("ffnOutB")), "ffnOut"]),
        _layernorm("lnF", d, 2, ["tmp", "ffnOut", _req(t.get("ffnNormW"), "ffnNormW"), _w(t.get("ffnNormB")),
                                 "mask", "x"]),
    ]


def pre_norm_layer(d: dict, t: dict, stream: str, first_norm: bool, attn_scale: float, window: int, rope: bool,
                   ffn: dict, rope_table_id: str = "cossin") -> list[dict]:
    """src/plan/layers.ts:164-204."""
    H, I = d["hidden"], d["intermediate"]
    ops: list[dict] = []
    if first_norm:
        ops.append(_layernorm("lnA", d, 0, [stream, "dummy", _req(t.get("attnNormW"), "attnNormW"),
                                            _w(t.get("attnNormB")), "mask", "normed"]))
    ops.append(_matmul("qkv", d, 3 * H, H, 0, ["normed" if first_norm else stream, _req(t.get("qkvW"), "qkvW"),
                                               _w(t.get("qkvB")), "qkv"]))
    if rope:
        ops.append({"name": "rope", "kernel": "rope", "constants": {"L": d["length"], "H": d["heads"], "D": d["headDim"]},
                    "bind": ["qkv", rope_table_id], "dispatch": ["rows", 2 * d["heads"]]})
    ops.extend(_standard_attention(d, attn_scale, window))
    ops.append(_matmul("attnOut", d, H, H, 0, ["ctx", _req(t.get("attnOutW"), "attnOutW"), _w(t.get("attnOutB")),
                                               "attnOut"]))
    ops.append(_add("addA", d, [stream, "attnOut"]))
    ops.append(_layernorm("lnF", d, 0, [stream, "dummy", _req(t.get("ffnNormW"), "ffnNormW"), _w(t.get("ffnNormB")),
                                        "mask", "normed"]))
    if ffn["kind"] == "geglu":
        ops.append(_matmul("ffnIn", d, 2 * I, H, 0, ["normed", _req(t.get("ffnInW"), "ffnInW"), _w(t.get("ffnInB")),
                                                     "mid"]))
        ops.append({"name": "geglu", "kernel": "geglu", "constants": {"I": I}, "bind": ["mid", "gate"],
                    "dispatch": ["rows", 1]})
        ops.append(_matmul("ffnOut", d, H, I, 0, ["gate", _req(t.get("ffnOutW"), "ffnOutW"), _w(t.get("ffnOutB")),
                                                  "ffnOut"]))
    else:
        ops.append(_matmul("lin1", d, ffn["width"], H, ffn["act"], ["normed", _req(t.get("ffnInW"), "ffnInW"),
                                                                    _w(t.get("ffnInB")), "mid"]))
        ops.append(_matmul("lin2", d, H, ffn["width"], 0, ["mid", _req(t.get("ffnOutW"), "ffnOutW"),
                                                           _w(t.get("ffnOutB")), "ffnOut"]))
    ops.append(_add("addF", d, [stream, "ffnOut"]))
    return ops


def _elements_written(op: dict) -> int:
    """src/plan/build.ts:98-107."""
    k, c = op["kernel"], op["constants"]
    if k in ("matmul", "mmtile", "mmtile16", "mmtile8", "layernorm", "embln", "pool"):
        return c["N"]
    if k == "geglu":
        return c["I"]
    if k in ("attention", "mbattention", "mbflash", "attpv"):
        return c["H"] * c["D"]
    if k == "gather":
        return c["D"]
    if k == "im2col":
        return c["N"] * c["KS"]
    return 0


def build_plan(spec: dict, head: dict, length: int, batch: int = 1, markers: int = 0, f16: bool = True,
               tensor_names=None) -> dict:
    """src/plan/build.ts:109-526: the encoder heads (classify, token, embed) and the marker
    heads (gliner2, julia: ``markers`` per sequence, or the Julia option count)."""
    names = tensor_names or tensor_names_for(spec["family"], spec)
    H = spec["hidden"]
    E = spec["embeddingSize"]

    def bytes_of(el: int) -> int:
        return math.ceil(el * (2 if f16 else 4) / 4) * 4

    M = length * batch
    pooled_head = head["type"] in ("classify", "token", "embed")
    if not pooled_head and head["type"] not in ("gliner2", "julia"):
        raise ValueError(f"head {head['type']} has no plan")
    markers = head["options"] if head["type"] == "julia" else 0 if pooled_head else markers
    K = markers * batch
    K16 = math.ceil(K / 16)
    eps = spec["block"]["norm"]["eps"]
    dims = {"hidden": H, "heads": spec["heads"], "headDim": spec["headDim"],
            "intermediate": spec["intermediate"], "rows": M, "length": length, "eps": eps}

    def ln(name, mode, bind, n=H, rows="rows"):
        return {"name": name, "kernel": "layernorm", "constants": {"N": n, "MODE": mode, "EPS": eps},
                "bind": bind, "dispatch": [rows, 1]}

    def mm(name, rows, n, k, act, bind, y_dim):
        return {"name": name, "kernel": "matmul", "constants": {"M": rows, "N": n, "K": k, "ACT": act},
                "bind": bind, "dispatch": [math.ceil(n / 16), y_dim]}

    segments: list[dict] = []
    slot = [0]

    def take(*bufs):
        out = []
        for b in bufs:
            out.append({"buffer": b, "slot": slot[0]})
            slot[0] += 1
        return out

    emb_w = f"w:{names.embedNormW}"
    emb_b = f"w:{names.embedNormB}" if names.embedNormB else "zero"
    embed = spec["embed"]
    absolute = embed["positions"] == "absolute"
    if absolute or embed["typeVocab"] > 0:
        type_table = "w:embeddings.type.weight" if embed["typeVocab"] > 0 else "zero"
        dst = "embE" if embed["project"] else "x"
        ops = [{"name": "embed", "kernel": "embln",
                "constants": {"N": E, "L": length, "OFFSET": embed["positionOffset"] if absolute else 0,
                              "MAXPOS": embed["maxPositions"] if absolute else 1, "EPS": embed["norm"]["eps"],
                              "MASKMUL": 1 if embed["maskMultiply"] else 0,
                              "POSIDS": 1 if embed.get("padId") is not None else 0},
                "bind": ["emb", "w:embeddings.position.weight" if absolute else "zero", type_table, "typeIds",
                         emb_w, emb_b, "mask", dst],
                "dispatch": ["rows", 1]}]
        if embed["project"]:
            ops.append(mm("project", M, H, E, 0, ["embE", "w:embeddings.project.weight",
                                                  "w:embeddings.project.bias", "x"], "rows16"))
        segments.append({"name": "embed", "prefix": "", "ops": ops, "capture": take("x")})
    elif embed["maskMultiply"]:
        segments.append({"name": "embed", "prefix": "",
                         "ops": [ln("embed", 1, ["emb", "dummy", emb_w, emb_b, "mask", "x"])],
                         "captureOps": [ln("embedPlain", 0, ["emb", "dummy", emb_w, emb_b, "mask", "tmp"])],
                         "capture": take("tmp", "x")})
    else:
        segments.append({"name": "embed", "prefix": "",
                         "ops": [ln("embed", 0, ["emb", "dummy", emb_w, emb_b, "mask", "x"])],
                         "capture": take("x")})

    conv = spec.get("conv")
    if conv:
        if not names.conv:
            raise ValueError("conv without tensor names")
        segments.append({"name": "convIn", "prefix": "ConvIn.", "ops": [
            {"name": "im2col", "kernel": "im2col", "constants": {"N": H, "L": length, "KS": conv["kernel"]},
             "bind": ["x", "mask", "cols"], "dispatch": ["rows", 1]},
            mm("conv", M, H, conv["kernel"] * H, act_code(conv["act"]),
               ["cols", f"w:{names.conv['w']}", f"w:{names.conv['b']}", "convOut"], "rows16"),
        ]})

    att = spec["attention"]
    rel = att.get("rel") if att["kind"] == "deberta-relative" else None
    if att["kind"] == "deberta-relative":
        if not rel:
            raise ValueError("deberta-relative attention needs attention.rel")
        rel_scale = math.sqrt((1 + len(rel["types"])) * (H / spec["heads"]))

        def attn_scale_of(l):
            return rel_scale, 0
    else:
        win = att.get("window")
        std_scale = (H / spec["heads"]) ** -0.5

        def attn_scale_of(l):
            return std_scale, (0 if not win or l % win["globalEvery"] == 0 else win["half"])
    rope = att.get("rope")
    rope_split = bool(rope) and rope["thetaGlobal"] != rope["thetaLocal"]
    for l in range(spec["layers"]):
        t = names.layer(l)
        scale, window = attn_scale_of(l)
        if spec["block"]["order"] == "post":
            rel_arg = None
            if rel:
                moff = rel_bucket_index(0, length - 1, rel["buckets"], rel["maxPositions"])
                rel_arg = {"moff": moff,
                           "nm": rel_bucket_index(length - 1, 0, rel["buckets"], rel["maxPositions"]) - moff + 1}
            ops = post_norm_layer(dims, t, act_code(spec["ffn"]["act"]), scale,
                                  att["kind"] == "standard", rel_arg)
        else:
            identity = spec["block"]["firstNormIdentity"] and l == 0
            ffn = ({"kind": "geglu"} if spec["ffn"]["kind"] == "geglu"
                   else {"kind": "mlp", "width": spec["intermediate"], "act": act_code(spec["ffn"]["act"])})
            tt = dict(t)
            if identity:
                tt.pop("attnNormW", None)
            ops = pre_norm_layer(dims, tt, "x", not identity, scale, window, bool(rope), ffn,
                                 ("cossinG" if window == 0 else "cossinL") if rope_split else "cossin")
        after_conv = l == 0 and bool(conv)
        seg = {"name": f"layer{l}", "prefix": f"L{l}.", "ops": ops, "skippable": True}
        if not after_conv:
            seg["capture"] = take("x")
        segments.append(seg)
        if after_conv and names.conv:
            segments.append({"name": "conv", "prefix": "Conv.", "ops": [
                {"name": "add", "kernel": "add", "constants": {"TOTAL": M * H, "N": H, "MODE": 0, "L": length},
                 "bind": ["convOut", "x"], "dispatch": [add_workgroups(M, H), 1]},
                ln("lnConv", 1, ["convOut", "dummy", f"w:{names.conv['normW']}", f"w:{names.conv['normB']}",
                                 "mask", "x"]),
            ], "capture": take("x")})

    stream = "x"
    if spec["block"]["finalNorm"]:
        if not names.finalNormW:
            raise ValueError("finalNorm without a tensor name")
        segments.append({"name": "final", "prefix": "", "ops": [
            ln("final", 0, ["x", "dummy", f"w:{names.finalNormW}",
                            f"w:{names.finalNormB}" if names.finalNormB else "zero", "mask", "tmp"])],
            "capture": take("tmp")})
        stream = "tmp"

    head_buffers: list[dict] = []
    need_first = False
    row_select = None
    out_buffer, out_rows, out_cols = "logits", K, 1
    if pooled_head:
        per_row = head["type"] == "token"
        rows = M if per_row else batch
        rows16 = "rows16" if per_row else math.ceil(batch / 16)
        prev = stream
        width = H
        ops = []
        if not per_row:
            pool = "first" if head.get("pool") == "cls" else head.get("pool")
            if pool == "first":
                need_first = True
                ops.append({"name": "gather", "kernel": "gather", "constants": {"K": 1, "D": H, "L": length},
                            "bind": ["first", stream, "states"], "dispatch": [1, 1]})
            else:
                ops.append({"name": "pool", "kernel": "pool",
                            "constants": {"L": length, "N": H, "MODE": 0 if pool == "mean" else 1},
                            "bind": [stream, "mask", "states"], "dispatch": [math.ceil(H / 64), batch]})
            head_buffers.append({"id": "states", "elements": batch * H, "final": False})
            prev = "states"
        steps = head["steps"]
        for i, step in enumerate(steps):
            last = i == len(steps) - 1
            dst = "out" if last else f"hd{i}"
            if step["op"] == "norm":
                ops.append({"name": f"step{i}", "kernel": "layernorm",
                            "constants": {"N": width, "MODE": 0, "EPS": step["eps"]},
                            "bind": [prev, "dummy", f"w:{step['name']}.weight",
                                     f"w:{step['name']}.bias" if step["bias"] else "zero", "mask", dst],
                            "dispatch": ["rows" if per_row else batch, 1]})
                head_buffers.append({"id": dst, "elements": rows * width, "final": last})
                prev = dst
                continue
            if step["in"] != width:
                raise ValueError(f"head step {step['name']}: input {step['in']}, previous width {width}")
            ops.append(mm(f"step{i}", rows, step["out"], step["in"], 0 if step["act"] == "none" else act_code(step["act"]),
                          [prev, f"w:{step['name']}.weight", f"w:{step['name']}.bias" if step["bias"] else "zero", dst],
                          rows16))
            head_buffers.append({"id": dst, "elements": rows * step["out"], "final": last})
            prev = dst
            width = step["out"]
        if not steps:
            if per_row:
                raise ValueError("a token head needs at least one dense step")
            next(b for b in head_buffers if b["id"] == "states")["final"] = True
        out_buffer, out_rows, out_cols = prev, rows, width
        segments.append({"name": "head", "prefix": "head.", "ops": ops})
    elif head["type"] == "gliner2":
        hh = head["hidden"]
        segments.append({"name": "head", "prefix": "head.", "ops": [
            {"name": "gather", "kernel": "gather", "constants": {"K": markers, "D": H, "L": length},
             "bind": ["packed", stream, "states"], "dispatch": [1, 1]},
            mm("fc1", K, hh, H, 1, ["states", "w:head.fc1.weight", "w:head.fc1.bias", "h1"], K16),
            mm("fc2", K, 1, hh, 0, ["h1", "w:head.fc2.weight", "w:head.fc2.bias", "raw"], K16),
            {"name": "maskl", "kernel": "masklogits", "constants": {"K": markers, "TEMP": head["temperature"]},
             "bind": ["raw", "packed", "logits"], "dispatch": [1, 1]},
        ]})
    else:
        if stream != "tmp":
            raise ValueError("julia head expects a final norm")
        segments.append({"name": "typed", "prefix": "", "ops": [
            {"name": "type", "kernel": "add", "constants": {"TOTAL": M * H, "N": H, "MODE": 1, "L": length},
             "bind": ["tmp", "typeRow"], "dispatch": [add_workgroups(M, H), 1]}], "capture": take("tmp")})
        row_select = {"table": "w:type_emb.weight", "dst": "typeRow", "rowBytes": bytes_of(H)}
        for i in range(head["layers"]):
            p = f"head.{i}"
            t = {"qkvW": f"{p}.in_proj.weight", "qkvB": f"{p}.in_proj.bias",
                 "attnOutW": f"{p}.out_proj.weight", "attnOutB": f"{p}.out_proj.bias",
                 "attnNormW": f"{p}.norm1.weight", "attnNormB": f"{p}.norm1.bias",
                 "ffnNormW": f"{p}.norm2.weight", "ffnNormB": f"{p}.norm2.bias",
                 "ffnInW": f"{p}.linear1.weight", "ffnInB": f"{p}.linear1.bias",
                 "ffnOutW": f"{p}.linear2.weight", "ffnOutB": f"{p}.linear2.bias"}
            segments.append({"name": f"head{i}", "prefix": f"head{i}.",
                             "ops": pre_norm_layer(dims, t, "tmp", True, (H / spec["heads"]) ** -0.5, 0, False,
                                                   {"kind": "mlp", "width": head["ffn"], "act": 1}),
                             "capture": take("tmp")})
        segments.append({"name": "scorer", "prefix": "scorer.", "ops": [
            {"name": "gather", "kernel": "gather", "constants": {"K": markers, "D": H, "L": length},
             "bind": ["packed", "tmp", "states"], "dispatch": [1, 1]},
            ln("ln", 0, ["states", "dummy", "w:scorer.norm.weight", "w:scorer.norm.bias", "mask", "kNormed"], H, K),
            mm("fc1", K, H, H, 2, ["kNormed", "w:scorer.fc1.weight", "w:scorer.fc1.bias", "h1"], K16),
            mm("fc2", K, 1, H, 0, ["h1", "w:scorer.fc2.weight", "w:scorer.fc2.bias", "raw"], K16),
            {"name": "maskl", "kernel": "masklogits", "constants": {"K": markers, "TEMP": 1.0},
             "bind": ["raw", "packed", "logits"], "dispatch": [1, 1]},
        ]})

    all_ops = [op for s in segments for op in s.get("captureOps", []) + s["ops"]]
    cols: dict[str, int] = {}
    for op in all_ops:
        dst = op["bind"][writable_bindings(op["kernel"], len(op["bind"]))[0]]
        n = _elements_written(op)
        if n > 0:
            cols[dst] = max(cols.get(dst, 0), n)
    k_rows = {"states", "kNormed", "h1", "raw"}
    decls: list[dict] = []

    def st(bid, nbytes, usage="rw", init=None):
        d = {"id": bid, "bytes": int(nbytes), "usage": usage}
        if init is not None:
            d["init"] = init
        decls.append(d)

    def rows_buf(bid, usage="rw"):
        c = cols.get(bid)
        if c is None:
            return
        st(bid, bytes_of((K if bid in k_rows else M) * c), usage)

    st("emb", bytes_of(M * E))
    if embed["project"]:
        st("embE", bytes_of(M * E))
    if absolute or embed["typeVocab"] > 0:
        st("typeIds", M * 4)
    for bid in ("x", "tmp"):
        if bid in cols:
            st(bid, bytes_of(M * cols[bid]), "rwSrc")
    if conv:
        st("cols", bytes_of(M * conv["kernel"] * H))
        st("convOut", bytes_of(M * H))
    for bid in ("normed", "qkv", "ctx", "attnOut", "mid", "gate", "ffnOut", "states", "kNormed", "h1", "raw"):
        if not (pooled_head and bid in k_rows):
            rows_buf(bid)
    st("mask", M * 4)
    if any("kinfo" in o["bind"] for o in all_ops):
        st("kinfo", 8 * batch)
    score_ops = [o for o in all_ops if o["kernel"] == "attscore"]
    for bid in ("c2p", "p2c"):
        rel_ops = [o for o in all_ops if o["kernel"] == "attrel" and o["bind"][4] == bid]
        if rel_ops:
            st(bid, max(o["constants"]["ROWS"] * o["constants"]["H"] * o["constants"]["NM"] * 4 for o in rel_ops))
    if score_ops:
        st("scores", max(o["constants"]["ROWS"] * o["constants"]["H"] * o["constants"]["L"] * 4 for o in score_ops))
    if any("dummy" in o["bind"] for o in all_ops):
        st("dummy", 4, "storage")
    if pooled_head:
        for b in head_buffers:
            st(b["id"], bytes_of(b["elements"]), "logits" if b["final"] else "rw")
        if need_first:
            st("first", 3 * batch * 4, "rw", np.zeros(3 * batch, dtype=np.uint32).tobytes())
    else:
        st("packed", 3 * K * 4)
        st("logits", K * 4, "logits")
    if rel:
        table = rel_pos_table(length, rel["buckets"], rel["maxPositions"])
        st("relidx", table.nbytes, "rw", table.tobytes())
    if rope and not rope_split:
        table = rope_table(length, rope["thetaGlobal"], spec["headDim"])
        st("cossin", table.nbytes, "rw", table.tobytes())
    elif rope:
        g = rope_table(length, rope["thetaGlobal"], spec["headDim"])
        lo = rope_table(length, rope["thetaLocal"], spec["headDim"])
        st("cossinG", g.nbytes, "rw", g.tobytes())
        st("cossinL", lo.nbytes, "rw", lo.tobytes())
    if row_select:
        st("typeRow", bytes_of(batch * H))
    zero_uses = [o for o in all_ops if "zero" in o["bind"]]
    if zero_uses:
        width_z = max(o["constants"]["N"] for o in zero_uses)
        st("zero", bytes_of(width_z), "rw", bytes(bytes_of(width_z)))

    validate_segments(segments, {d["id"] for d in decls})
    inputs = {"embeddings": "emb", "mask": "mask"}
    if not pooled_head:
        inputs["markers"] = "packed"
    elif absolute or embed["typeVocab"] > 0:
        inputs["typeIds"] = "typeIds"
    plan = {
        "f16": f16, "length": length, "batch": batch, "markers": markers, "embeddingSize": E,
        "buffers": decls, "segments": segments, "inputs": inputs,
        "output": ({"buffer": out_buffer, "bytes": bytes_of(out_rows * out_cols), "dtype": "storage",
                    "rows": out_rows, "cols": out_cols} if pooled_head else
                   {"buffer": "logits", "bytes": K * 4, "dtype": "f32", "rows": K, "cols": 1}),
        "captureSlots": slot[0], "captureSlotBytes": length * H * 4,
    }
    if row_select:
        plan["rowSelect"] = row_select
    return plan


def plan_to_json(plan: dict) -> str:
    """The Plan as JSON for the C ABI: buffer ``init`` blobs become base64 strings under
    ``init_b64`` (``src/plan/ir.ts:17`` keeps them as typed arrays)."""
    def conv(o: Any):
        if isinstance(o, dict):
            out = {}
            for k, v in o.items():
                if k == "init":
                    out["init_b64"] = base64.b64encode(bytes(v)).decode("ascii")
                else:
                    out[k] = conv(v)
            return out
        if isinstance(o, list):
            return [conv(v) for v in o]
        if isinstance(o, (np.integer,)):
            return int(o)
        if isinstance(o, (np.floating,)):
            return float(o)
        return o
    return json.dumps(conv(plan), separators=(",", ":"))


def plan_ops(plan: dict) -> list[dict]:
    return [op for s in plan["segments"] for op in s["ops"]]

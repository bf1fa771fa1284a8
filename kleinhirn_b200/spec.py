"""Model description: Hugging Face ``config.json`` -> ModelSpec + HeadSpec.

Host-side restatement of kleinhirn's model description layer so that the CUDA backend and
its tests can build the same Plans the TypeScript engine builds:

- ``spec_from_hf_config`` follows ``src/plan/hf.ts:179-258`` (BERT, ELECTRA, RoBERTa, XLM-R,
  DistilBERT), ``src/plan/hf.ts:282-365`` (DeBERTa-v2/v3) and ``src/plan/hf.ts:395-458``
  (ModernBERT). Every unsupported value raises ``ValueError`` naming the config key, like
  ``fail()`` in ``src/plan/hf.ts:39-41``.
- ``tensor_names_for`` follows ``src/plan/spec.ts:109-183``.
- ``position_rows`` follows ``src/plan/spec.ts:63-66``.

Specs and heads are plain dicts with the field names of the TypeScript interfaces
(``ModelSpec`` ``src/plan/spec.ts:12-58``, ``HeadSpec`` ``src/plan/spec.ts:74-85``), so they
serialise to the same JSON the reference writes into a manifest's ``spec`` and ``head``.
"""
from __future__ import annotations

import math
from typing import Any

ACTS = ("gelu", "relu", "tanh", "silu")
FAMILIES = ("bert", "electra", "roberta", "xlm-roberta", "distilbert", "deberta-v2", "modernbert")
ST_ACTS = {
    "torch.nn.modules.activation.Tanh": "tanh",
    "torch.nn.modules.activation.ReLU": "relu",
    "torch.nn.modules.activation.GELU": "gelu",
    "torch.nn.modules.activation.SiLU": "silu",
    "torch.nn.modules.linear.Identity": "none",
}
PROBLEMS = {
    "single_label_classification": "single",
    "multi_label_classification": "multi",
    "regression": "regression",
}


def fail(key: str, why: str):
    """src/plan/hf.ts:39-41: every rejection names the config key."""
    raise ValueError(f"config key '{key}': {why}")


def _num(config: dict, key: str, fallback: float | None = None) -> float:
    v = config.get(key, fallback)
    if v is None:
        v = fallback
    if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v):
        fail(key, f"expected a number, got {v}")
    return v


def _bool(config: dict, key: str, fallback: bool) -> bool:
    v = config.get(key, fallback)
    if v is None:
        v = fallback
    if not isinstance(v, bool):
        fail(key, f"expected a boolean, got {v}")
    return v


def _act_of(config: dict, key: str, fallback: str) -> str:
    act = config.get(key, fallback)
    if act is None:
        act = fallback
    if act not in ACTS:
        fail(key, f"'{config.get(key)}' is outside {', '.join(ACTS)}")
    return act


def position_rows(pad_id: int, ids) -> list[int]:
    """src/plan/spec.ts:63-66: a pad id keeps row padId, every other id gets padId plus the
    number of non-pad ids up to and including it (transformers'
    create_position_ids_from_input_ids)."""
    out = []
    count = 0
    for i in ids:
        if i == pad_id:
            out.append(pad_id)
        else:
            count += 1
            out.append(pad_id + count)
    return out


def _pool_from_st(pooling: dict | None) -> str:
    if not pooling:
        fail("pooling", "embeddings need the 1_Pooling/config.json content")
    modes = [k for k, v in pooling.items() if k.startswith("pooling_mode_") and v is True]
    if len(modes) != 1:
        fail("pooling_mode", f"exactly one mode expected, got [{', '.join(modes)}]")
    return {"pooling_mode_mean_tokens": "mean", "pooling_mode_cls_token": "cls",
            "pooling_mode_max_tokens": "max"}.get(modes[0]) or fail(modes[0], "pooling mode is not supported")


def _dense_steps(extras: dict, hidden: int) -> list[dict]:
    """src/plan/hf.ts:61-75 (sentence-transformers Dense modules)."""
    dense = (extras.get("sentenceTransformers") or {}).get("dense")
    if dense is True:
        fail("dense", "the Dense module config (2_Dense/config.json) is missing")
    if not dense:
        return []
    width = hidden
    steps = []
    for i, d in enumerate(dense):
        act = ST_ACTS.get(d["activation_function"])
        if act is None:
            fail("activation_function", f"'{d['activation_function']}' is not supported")
        if d["in_features"] != width:
            fail("in_features", f"Dense {i} expects {d['in_features']}, input is {width}")
        width = d["out_features"]
        steps.append({"op": "dense", "name": f"head.dense{i}", "in": d["in_features"],
                      "out": d["out_features"], "act": act, "bias": d["bias"]})
    return steps


def _embed_head(extras: dict, hidden: int) -> dict:
    st = extras.get("sentenceTransformers") or {}
    return {"type": "embed", "pool": _pool_from_st(st.get("pooling")),
            "steps": _dense_steps(extras, hidden), "normalize": st.get("normalize") is True}


def _class_count(config: dict, task: str) -> int:
    id2label = config.get("id2label")
    classes = len(id2label) if id2label else int(_num(config, "num_labels", 2))
    if task == "reranking" and classes != 1:
        fail("id2label", f"reranking needs one logit, got {classes}")
    if task == "nli":
        entail = [n for n in (id2label or {}).values() if n.lower().startswith("entail")]
        if len(entail) != 1:
            fail("id2label", 'NLI needs exactly one label starting with "entail"')
    return classes


def _problem_of(config: dict, classes: int) -> dict:
    raw = config.get("problem_type")
    if raw is None:
        return {}
    problem = PROBLEMS.get(raw) if isinstance(raw, str) else None
    if not problem:
        fail("problem_type", f"'{raw}' is outside {', '.join(PROBLEMS)}")
    return {} if problem == ("regression" if classes == 1 else "single") else {"problem": problem}


def _roberta_offset(config: dict, template) -> int:
    """src/plan/hf.ts:116-125."""
    pad = int(_num(config, "pad_token_id", 1))
    if not template:
        fail("tokenizer template", "RoBERTa and XLM-R need the single template of tokenizer.json for the position offset")
    if any(t is not None and t == pad for t in template[1:]):
        fail("pad_token_id", f"{pad} is the id of a later special token of the single template")
    return pad if template[0] == pad else pad + 1


def _dense(name: str, i: int, o: int, a: str) -> dict:
    return {"op": "dense", "name": name, "in": i, "out": o, "act": a, "bias": True}


def spec_from_hf_config(config: dict, extras: dict) -> tuple[dict, dict, str]:
    """src/plan/hf.ts:179-258."""
    model_type = config.get("model_type")
    if model_type not in FAMILIES:
        fail("model_type", f"'{model_type}' is not in the covered rows ({', '.join(FAMILIES)})")
    if model_type == "deberta-v2":
        return _spec_from_deberta(config, extras)
    if model_type == "modernbert":
        return _spec_from_modernbert(config, extras)
    if config.get("is_decoder") is True and model_type != "distilbert":
        fail("is_decoder", "true: causal attention is not planned")
    if config.get("add_cross_attention") is True and model_type != "distilbert":
        fail("add_cross_attention", "true: cross-attention is not planned")
    position_type = config.get("position_embedding_type") or "absolute"
    if position_type != "absolute":
        fail("position_embedding_type", f"'{position_type}', only 'absolute' is planned")
    act_key = "activation" if model_type == "distilbert" else "hidden_act"
    act = config.get(act_key) or "gelu"
    if act not in ACTS:
        fail(act_key, f"'{config.get(act_key)}' is outside {', '.join(ACTS)}")
    if model_type == "distilbert":
        hidden, layers, heads = int(_num(config, "dim")), int(_num(config, "n_layers")), int(_num(config, "n_heads"))
        intermediate = int(_num(config, "hidden_dim"))
        eps, type_vocab, position_offset = 1e-12, 0, 0
        sinusoidal = config.get("sinusoidal_pos_embds") is True
    else:
        hidden = int(_num(config, "hidden_size"))
        layers = int(_num(config, "num_hidden_layers"))
        heads = int(_num(config, "num_attention_heads"))
        intermediate = int(_num(config, "intermediate_size"))
        eps = _num(config, "layer_norm_eps", 1e-12)
        type_vocab = int(_num(config, "type_vocab_size", 2))
        position_offset = (_roberta_offset(config, extras.get("template"))
                           if model_type in ("roberta", "xlm-roberta") else 0)
        sinusoidal = False
    hidden_key = "dim" if model_type == "distilbert" else "hidden_size"
    heads_key = "n_heads" if model_type == "distilbert" else "num_attention_heads"
    if hidden % heads != 0:
        fail(heads_key, f"{heads} does not divide {hidden_key} {hidden}")
    head_dim = hidden // heads
    if head_dim > 64:
        fail(f"{hidden_key} / {heads_key}", f"head dimension {head_dim} exceeds 64")
    embedding_size = int(_num(config, "embedding_size", hidden)) if model_type == "electra" else hidden
    norm = {"eps": eps, "bias": True}
    max_positions = int(_num(config, "max_position_embeddings", 512))
    if max_positions <= position_offset:
        fail("max_position_embeddings", f"{max_positions} rows leave no position after the offset {position_offset}")
    embed = {"positions": "absolute", "positionOffset": position_offset, "maxPositions": max_positions}
    if model_type in ("roberta", "xlm-roberta"):
        embed["padId"] = int(_num(config, "pad_token_id", 1))
    embed.update({"typeVocab": type_vocab, "norm": norm, "maskMultiply": False,
                  "project": model_type == "electra" and embedding_size != hidden})
    if sinusoidal:
        embed["sinusoidal"] = True
    spec = {
        "family": model_type, "hidden": hidden, "layers": layers, "heads": heads, "headDim": head_dim,
        "intermediate": intermediate, "vocab": int(_num(config, "vocab_size")), "embeddingSize": embedding_size,
        "embed": embed,
        "attention": {"kind": "standard", "bias": True, "scale": head_dim ** -0.5},
        "block": {"order": "post", "firstNormIdentity": False, "finalNorm": False, "norm": norm},
        "ffn": {"kind": "mlp", "act": act, "bias": True},
    }
    task = extras["task"]
    if task == "embeddings":
        head = _embed_head(extras, hidden)
    else:
        classes = _class_count(config, task)
        if task == "token-classification":
            head = {"type": "token", "steps": [_dense("head.classifier", hidden, classes, "none")], "classes": classes}
        else:
            first = {"electra": ("head.dense", "gelu", "head.out_proj"),
                     "roberta": ("head.dense", "tanh", "head.out_proj"),
                     "xlm-roberta": ("head.dense", "tanh", "head.out_proj"),
                     "distilbert": ("head.pre_classifier", "relu", "head.classifier")}.get(
                         model_type, ("head.pooler", "tanh", "head.classifier"))
            head = {"type": "classify", "pool": "first", "classes": classes, **_problem_of(config, classes),
                    "steps": [_dense(first[0], hidden, hidden, first[1]),
                              _dense(first[2], hidden, classes, "none")]}
    return spec, head, task


def _spec_from_deberta(config: dict, extras: dict) -> tuple[dict, dict, str]:
    """src/plan/hf.ts:282-365."""
    hidden = int(_num(config, "hidden_size"))
    layers = int(_num(config, "num_hidden_layers"))
    heads = int(_num(config, "num_attention_heads"))
    if hidden % heads != 0:
        fail("num_attention_heads", f"{heads} does not divide hidden_size {hidden}")
    head_dim = hidden // heads
    if head_dim > 64:
        fail("hidden_size / num_attention_heads", f"head dimension {head_dim} exceeds 64")
    if config.get("attention_head_size") is not None and config["attention_head_size"] != head_dim:
        fail("attention_head_size", f"{config['attention_head_size']} differs from hidden_size / num_attention_heads")
    conv_kernel = int(_num(config, "conv_kernel_size", 0))
    if conv_kernel > 0:
        if conv_kernel % 2 != 1:
            fail("conv_kernel_size", f"{conv_kernel}, only odd kernels keep the length")
        if _num(config, "conv_groups", 1) != 1:
            fail("conv_groups", "grouped convolution is not planned")
    embedding_size = int(_num(config, "embedding_size", hidden))
    if embedding_size != hidden:
        fail("embedding_size", f"{embedding_size} differs from hidden_size {hidden}")
    act = _act_of(config, "hidden_act", "gelu")
    eps = _num(config, "layer_norm_eps", 1e-7)
    norm = {"eps": eps, "bias": True}
    max_positions = int(_num(config, "max_position_embeddings", 512))
    position_biased = _bool(config, "position_biased_input", True)
    relative = _bool(config, "relative_attention", False)
    if relative:
        if not _bool(config, "share_att_key", False):
            fail("share_att_key", "false: separate position projections are not planned")
        norms = [x.strip() for x in str(config.get("norm_rel_ebd") or "none").lower().split("|")]
        if norms != ["layer_norm"]:
            fail("norm_rel_ebd", f"'{config.get('norm_rel_ebd')}', only 'layer_norm' is planned")
        types = config.get("pos_att_type")
        if not isinstance(types, list) or len(types) != 2 or "p2c" not in types or "c2p" not in types:
            fail("pos_att_type", f"{types}, the kernel needs exactly c2p and p2c")
        buckets = int(_num(config, "position_buckets", -1))
        if buckets <= 0:
            fail("position_buckets", f"{buckets}, relative positions without buckets are not planned")
        rel = int(_num(config, "max_relative_positions", -1))
        attention = {"kind": "deberta-relative", "bias": True, "scale": 1 / math.sqrt(3 * head_dim),
                     "rel": {"buckets": buckets, "maxPositions": rel if rel > 0 else max_positions,
                             "types": ["c2p", "p2c"]}}
    else:
        attention = {"kind": "standard", "bias": True, "scale": head_dim ** -0.5}
    if not relative and not position_biased:
        fail("position_biased_input", "false without relative attention leaves no position signal")
    spec = {
        "family": "deberta-v2", "hidden": hidden, "layers": layers, "heads": heads, "headDim": head_dim,
        "intermediate": int(_num(config, "intermediate_size")), "vocab": int(_num(config, "vocab_size")),
        "embeddingSize": embedding_size,
        "embed": {"positions": "absolute" if position_biased else "none", "positionOffset": 0,
                  "maxPositions": max_positions, "typeVocab": int(_num(config, "type_vocab_size", 0)),
                  "norm": norm, "maskMultiply": True, "project": False},
        "attention": attention,
        "block": {"order": "post", "firstNormIdentity": False, "finalNorm": False, "norm": norm},
        "ffn": {"kind": "mlp", "act": act, "bias": True},
    }
    if conv_kernel > 0:
        spec["conv"] = {"kernel": conv_kernel, "act": _act_of(config, "conv_act", "tanh")}
    task = extras["task"]
    if task == "embeddings":
        return spec, _embed_head(extras, hidden), task
    classes = _class_count(config, task)
    if task == "token-classification":
        return spec, {"type": "token", "steps": [_dense("head.classifier", hidden, classes, "none")],
                      "classes": classes}, task
    pooler_size = int(_num(config, "pooler_hidden_size", 768))
    if pooler_size != hidden:
        fail("pooler_hidden_size", f"{pooler_size} differs from hidden_size {hidden}")
    pooler_act = _act_of(config, "pooler_hidden_act", "gelu")
    head = {"type": "classify", "pool": "first", "classes": classes, **_problem_of(config, classes),
            "steps": [_dense("head.pooler", hidden, hidden, pooler_act),
                      _dense("head.classifier", hidden, classes, "none")]}
    return spec, head, task


def _modernbert_thetas(config: dict) -> tuple[float, float]:
    """src/plan/hf.ts:369-392."""
    if config.get("rope_scaling") is not None:
        fail("rope_scaling", "scaled RoPE is not planned")
    params = config.get("rope_parameters")
    if params and not params.get("full_attention") and not params.get("sliding_attention"):
        fail("rope_parameters", "expected an entry per layer type (full_attention, sliding_attention)")

    def theta(kind: str, legacy: str, fallback: float) -> float:
        entry = (params or {}).get(kind)
        if entry:
            rope_type = entry.get("rope_type", "default")
            if rope_type != "default":
                fail(f"rope_parameters.{kind}.rope_type", f"'{rope_type}', only 'default' is planned")
            extra = [k for k in entry if k not in ("rope_type", "rope_theta")]
            if extra:
                fail(f"rope_parameters.{kind}", f"key {extra[0]} is not planned")
            if entry.get("rope_theta") is not None:
                return _num(entry, "rope_theta")
        return _num(config, legacy, fallback)

    return theta("full_attention", "global_rope_theta", 160000), theta("sliding_attention", "local_rope_theta", 10000)


def _spec_from_modernbert(config: dict, extras: dict) -> tuple[dict, dict, str]:
    """src/plan/hf.ts:395-458."""
    hidden = int(_num(config, "hidden_size"))
    layers = int(_num(config, "num_hidden_layers"))
    heads = int(_num(config, "num_attention_heads"))
    if hidden % heads != 0:
        fail("num_attention_heads", f"{heads} does not divide hidden_size {hidden}")
    head_dim = hidden // heads
    if head_dim > 64:
        fail("hidden_size / num_attention_heads", f"head dimension {head_dim} exceeds 64")
    if head_dim % 2 != 0:
        fail("hidden_size / num_attention_heads", f"head dimension {head_dim} is odd, RoPE rotates pairs")
    if config.get("is_causal") is True:
        fail("is_causal", "causal attention is not planned")
    if config.get("causal_mask") is True:
        fail("causal_mask", "causal attention is not planned")
    mlp_act = config.get("hidden_activation") or "gelu"
    if mlp_act != "gelu":
        fail("hidden_activation", f"'{mlp_act}', the GeGLU kernel computes gelu")
    eps = _num(config, "norm_eps", 1e-5)
    norm_bias = _bool(config, "norm_bias", False)
    attention_bias = _bool(config, "attention_bias", False)
    mlp_bias = _bool(config, "mlp_bias", False)
    norm = {"eps": eps, "bias": norm_bias}
    every = int(_num(config, "global_attn_every_n_layers", 3))
    if every < 1:
        fail("global_attn_every_n_layers", f"{every}")
    local = int(_num(config, "local_attention", 128))
    types = config.get("layer_types")
    if types is not None:
        want = ["sliding_attention" if i % every else "full_attention" for i in range(layers)]
        if list(types) != want:
            fail("layer_types", "differs from the pattern of global_attn_every_n_layers")
    theta_g, theta_l = _modernbert_thetas(config)
    spec = {
        "family": "modernbert", "hidden": hidden, "layers": layers, "heads": heads, "headDim": head_dim,
        "intermediate": int(_num(config, "intermediate_size")), "vocab": int(_num(config, "vocab_size")),
        "embeddingSize": hidden,
        "embed": {"positions": "none", "positionOffset": 0,
                  "maxPositions": int(_num(config, "max_position_embeddings", 8192)),
                  "typeVocab": 0, "norm": norm, "maskMultiply": False, "project": False},
        "attention": {"kind": "standard", "bias": attention_bias, "scale": head_dim ** -0.5,
                      "rope": {"thetaGlobal": theta_g, "thetaLocal": theta_l},
                      "window": {"half": local // 2, "globalEvery": every}},
        "block": {"order": "pre", "firstNormIdentity": True, "finalNorm": True, "norm": norm},
        "ffn": {"kind": "geglu", "act": "gelu", "bias": mlp_bias},
    }
    task = extras["task"]
    if task == "embeddings":
        return spec, _embed_head(extras, hidden), task
    classes = _class_count(config, task)
    steps = [
        {"op": "dense", "name": "head.dense", "in": hidden, "out": hidden,
         "act": _act_of(config, "classifier_activation", "gelu"), "bias": _bool(config, "classifier_bias", False)},
        {"op": "norm", "name": "head.norm", "eps": eps, "bias": norm_bias},
        {"op": "dense", "name": "head.classifier", "in": hidden, "out": classes, "act": "none", "bias": True},
    ]
    if task == "token-classification":
        return spec, {"type": "token", "steps": steps, "classes": classes}, task
    pooling = config.get("classifier_pooling") or "cls"
    if pooling not in ("cls", "mean"):
        fail("classifier_pooling", f"'{pooling}', expected cls or mean")
    return spec, {"type": "classify", "pool": "first" if pooling == "cls" else "mean", "steps": steps,
                  "classes": classes, **_problem_of(config, classes)}, task


class TensorNames:
    """src/plan/spec.ts:99-107: the tensor names one family reads."""

    def __init__(self, embed_norm_w: str, embed_norm_b: str | None, layer, final_norm_w: str | None = None,
                 final_norm_b: str | None = None, conv: dict | None = None):
        self.embedNormW = embed_norm_w
        self.embedNormB = embed_norm_b
        self.finalNormW = final_norm_w
        self.finalNormB = final_norm_b
        self.layer = layer
        self.conv = conv


def _deberta_layer(l: int) -> dict:
    return {
        "qkvW": f"layers.{l}.qkv.weight", "qkvB": f"layers.{l}.qkv.bias",
        "posKey": f"layers.{l}.pos_key", "posQuery": f"layers.{l}.pos_query",
        "attnOutW": f"layers.{l}.attn_out.weight", "attnOutB": f"layers.{l}.attn_out.bias",
        "attnNormW": f"layers.{l}.attn_ln.weight", "attnNormB": f"layers.{l}.attn_ln.bias",
        "ffnInW": f"layers.{l}.ffn_in.weight", "ffnInB": f"layers.{l}.ffn_in.bias",
        "ffnOutW": f"layers.{l}.ffn_out.weight", "ffnOutB": f"layers.{l}.ffn_out.bias",
        "ffnNormW": f"layers.{l}.ffn_ln.weight", "ffnNormB": f"layers.{l}.ffn_ln.bias",
    }


def _bert_layer(l: int) -> dict:
    t = _deberta_layer(l)
    del t["posKey"], t["posQuery"]
    return t


DEBERTA_CONV_TENSORS = {"w": "conv.weight", "b": "conv.bias", "normW": "conv.ln.weight", "normB": "conv.ln.bias"}


def modernbert_tensors(attention: bool, mlp: bool, norm: bool) -> TensorNames:
    """src/plan/spec.ts:142-159."""
    def layer(l: int) -> dict:
        t = {"qkvW": f"layers.{l}.wqkv.weight", "attnOutW": f"layers.{l}.attn_out.weight",
             "attnNormW": f"layers.{l}.attn_norm.weight", "ffnInW": f"layers.{l}.mlp_in.weight",
             "ffnOutW": f"layers.{l}.mlp_out.weight", "ffnNormW": f"layers.{l}.mlp_norm.weight"}
        if attention:
            t["qkvB"] = f"layers.{l}.wqkv.bias"
            t["attnOutB"] = f"layers.{l}.attn_out.bias"
        if mlp:
            t["ffnInB"] = f"layers.{l}.mlp_in.bias"
            t["ffnOutB"] = f"layers.{l}.mlp_out.bias"
        if norm:
            t["attnNormB"] = f"layers.{l}.attn_norm.bias"
            t["ffnNormB"] = f"layers.{l}.mlp_norm.bias"
        return t
    return TensorNames("embeddings.norm.weight", "embeddings.norm.bias" if norm else None, layer,
                       "final_norm.weight", "final_norm.bias" if norm else None)


def tensor_names_for(family: str, spec: dict | None = None) -> TensorNames:
    """src/plan/spec.ts:171-183."""
    if family in ("bert", "electra", "roberta", "xlm-roberta", "distilbert"):
        return TensorNames("embeddings.LayerNorm.weight", "embeddings.LayerNorm.bias", _bert_layer)
    if family == "deberta-v2":
        return TensorNames("embeddings.LayerNorm.weight", "embeddings.LayerNorm.bias", _deberta_layer,
                           conv=DEBERTA_CONV_TENSORS if spec and spec.get("conv") else None)
    if family == "modernbert":
        if spec is None:
            return modernbert_tensors(False, False, False)
        return modernbert_tensors(spec["attention"]["bias"], spec["ffn"]["bias"], spec["block"]["norm"]["bias"])
    raise ValueError(f"no tensor names for family {family}")


def output_cols(spec: dict, head: dict) -> int:
    """Output columns of an encoder head (src/encoder.ts:318-328)."""
    if head["type"] in ("classify", "token"):
        return head["classes"]
    if head["type"] == "embed":
        width = spec["hidden"]
        for s in head["steps"]:
            if s["op"] == "dense":
                width = s["out"]
        return width
    raise ValueError(f"head {head['type']} is not an encoder head")


def manifest_tensor_shapes(spec: dict, head: dict) -> dict[str, tuple[int, ...]]:
    """Canonical tensor names and shapes of a converted model (the names of
    src/convert/names.ts:127-293 after conversion: fused QKV [3H, H], weights [out, in],
    DeBERTa pos_key/pos_query [2 * buckets, H]). The word table is included; it stays on the
    host (src/backend.ts:51-56)."""
    H, E, I = spec["hidden"], spec["embeddingSize"], spec["intermediate"]
    names = tensor_names_for(spec["family"], spec)
    out: dict[str, tuple[int, ...]] = {"embeddings.word.weight": (spec["vocab"], E)}
    emb = spec["embed"]
    if emb["positions"] == "absolute":
        out["embeddings.position.weight"] = (emb["maxPositions"], E)
    if emb["typeVocab"] > 0:
        out["embeddings.type.weight"] = (emb["typeVocab"], E)
    out[names.embedNormW] = (E,)
    if names.embedNormB:
        out[names.embedNormB] = (E,)
    if emb["project"]:
        out["embeddings.project.weight"] = (H, E)
        out["embeddings.project.bias"] = (H,)
    if spec.get("conv"):
        k = spec["conv"]["kernel"]
        out["conv.weight"] = (H, k * H)
        out["conv.bias"] = (H,)
        out["conv.ln.weight"] = (H,)
        out["conv.ln.bias"] = (H,)
    ffn_in = 2 * I if spec["ffn"]["kind"] == "geglu" else I
    for l in range(spec["layers"]):
        t = names.layer(l)
        if spec["block"]["firstNormIdentity"] and l == 0:
            t = {k: v for k, v in t.items() if k not in ("attnNormW", "attnNormB")}
        shapes = {"qkvW": (3 * H, H), "qkvB": (3 * H,), "attnOutW": (H, H), "attnOutB": (H,),
                  "attnNormW": (H,), "attnNormB": (H,), "ffnInW": (ffn_in, H), "ffnInB": (ffn_in,),
                  "ffnOutW": (H, I), "ffnOutB": (H,), "ffnNormW": (H,), "ffnNormB": (H,)}
        if spec["attention"]["kind"] == "deberta-relative":
            rows = 2 * spec["attention"]["rel"]["buckets"]
            shapes["posKey"] = (rows, H)
            shapes["posQuery"] = (rows, H)
        for k, name in t.items():
            out[name] = shapes[k]
    if names.finalNormW:
        out[names.finalNormW] = (H,)
        if names.finalNormB:
            out[names.finalNormB] = (H,)
    if head["type"] in ("gliner2", "julia"):
        out.update(marker_head_tensor_shapes(spec, head))
    if head["type"] in ("classify", "token", "embed"):
        for s in head["steps"]:
            if s["op"] == "norm":
                out[f"{s['name']}.weight"] = (H,)
                if s["bias"]:
                    out[f"{s['name']}.bias"] = (H,)
            else:
                out[f"{s['name']}.weight"] = (s["out"], s["in"])
                if s["bias"]:
                    out[f"{s['name']}.bias"] = (s["out"],)
    return out


def spec_from_gliner_manifest(enc: dict, head: dict, markers: int = 16) -> tuple[dict, dict]:
    """src/plan/spec.ts:212-246: the GLiNER2 span classifier, a DeBERTa-v3 encoder (relative
    attention, no absolute positions, no type table) and the marker head. ``enc`` holds the
    manifest ``encoder`` fields (hiddenSize, layers, heads, intermediateSize, positionBuckets,
    maxRelativePositions, layerNormEps, vocabSize); ``head`` temperature and hiddenSize."""
    head_dim = enc["hiddenSize"] // enc["heads"]
    norm = {"eps": enc["layerNormEps"], "bias": True}
    spec = {
        "family": "deberta-v2", "hidden": enc["hiddenSize"], "layers": enc["layers"], "heads": enc["heads"],
        "headDim": head_dim, "intermediate": enc["intermediateSize"], "vocab": enc.get("vocabSize") or 0,
        "embeddingSize": enc["hiddenSize"],
        "embed": {"positions": "none", "positionOffset": 0, "maxPositions": 0, "typeVocab": 0, "norm": norm,
                  "maskMultiply": True, "project": False},
        "attention": {"kind": "deberta-relative", "bias": True, "scale": 1 / math.sqrt(3 * head_dim),
                      "rel": {"buckets": enc["positionBuckets"], "maxPositions": enc["maxRelativePositions"],
                              "types": ["c2p", "p2c"]}},
        "block": {"order": "post", "firstNormIdentity": False, "finalNorm": False, "norm": norm},
        "ffn": {"kind": "mlp", "act": "gelu", "bias": True},
    }
    return spec, {"type": "gliner2", "hidden": int(head.get("hiddenSize") or 768),
                  "temperature": head["temperature"], "markers": markers}


def spec_from_julia_manifest(enc: dict) -> tuple[dict, dict]:
    """src/plan/spec.ts:248-276: Julia, a ModernBERT encoder without biases (RoPE, local
    windows) and the typed head (type row, pre-norm head layers, marker scorer). ``enc`` holds
    layers, hiddenSize, heads, intermediate, normEps, ropeTheta, localAttention, globalEvery,
    headLayers, headFfn, options, maxPos, vocab."""
    head_dim = enc["hiddenSize"] // enc["heads"]
    norm = {"eps": enc["normEps"], "bias": False}
    spec = {
        "family": "modernbert", "hidden": enc["hiddenSize"], "layers": enc["layers"], "heads": enc["heads"],
        "headDim": head_dim, "intermediate": enc["intermediate"], "vocab": enc.get("vocab") or 0,
        "embeddingSize": enc["hiddenSize"],
        "embed": {"positions": "none", "positionOffset": 0, "maxPositions": enc.get("maxPos") or 0, "typeVocab": 0,
                  "norm": norm, "maskMultiply": False, "project": False},
        "attention": {"kind": "standard", "bias": False, "scale": head_dim ** -0.5,
                      "rope": {"thetaGlobal": enc["ropeTheta"], "thetaLocal": enc["ropeTheta"]},
                      "window": {"half": enc["localAttention"], "globalEvery": enc["globalEvery"]}},
        "block": {"order": "pre", "firstNormIdentity": True, "finalNorm": True, "norm": norm},
        "ffn": {"kind": "geglu", "act": "gelu", "bias": False},
    }
    return spec, {"type": "julia", "layers": enc["headLayers"], "ffn": enc["headFfn"], "options": enc["options"]}


def marker_head_tensor_shapes(spec: dict, head: dict, qtypes: int = 3) -> dict[str, tuple[int, ...]]:
    """Tensors of the marker heads (src/plan/build.ts:358-430): GLiNER2 fc1/fc2; Julia's type
    table (``qtypes`` rows), head layers (nn.TransformerEncoderLayer names) and scorer."""
    H = spec["hidden"]
    if head["type"] == "gliner2":
        hh = head["hidden"]
        return {"head.fc1.weight": (hh, H), "head.fc1.bias": (hh,), "head.fc2.weight": (1, hh),
                "head.fc2.bias": (1,)}
    if head["type"] != "julia":
        raise ValueError(f"head {head['type']} is not a marker head")
    out: dict[str, tuple[int, ...]] = {"type_emb.weight": (qtypes, H)}
    F = head["ffn"]
    for i in range(head["layers"]):
        p = f"head.{i}"
        out.update({f"{p}.in_proj.weight": (3 * H, H), f"{p}.in_proj.bias": (3 * H,),
                    f"{p}.out_proj.weight": (H, H), f"{p}.out_proj.bias": (H,),
                    f"{p}.norm1.weight": (H,), f"{p}.norm1.bias": (H,),
                    f"{p}.norm2.weight": (H,), f"{p}.norm2.bias": (H,),
                    f"{p}.linear1.weight": (F, H), f"{p}.linear1.bias": (F,),
                    f"{p}.linear2.weight": (H, F), f"{p}.linear2.bias": (H,)})
    out.update({"scorer.norm.weight": (H,), "scorer.norm.bias": (H,), "scorer.fc1.weight": (H, H),
                "scorer.fc1.bias": (H,), "scorer.fc2.weight": (1, H), "scorer.fc2.bias": (1,)})
    return out

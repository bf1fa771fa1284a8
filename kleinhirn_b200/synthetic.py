"""The five benchmark configurations, random-init weights and seeded synthetic inputs.

There is no network and no checkpoint: every model is a random-init encoder of the named
architecture (linear weights N(0, 0.02), biases N(0, 0.02), LayerNorm weights 1 + N(0, 0.02)),
converted the way the reference's converter converts a checkpoint (fused QKV [3H, H], weights
[out, in] as PyTorch stores them, src/convert/names.ts:5,217-236; DeBERTa pos_key / pos_query
= projection of LayerNorm(rel_embeddings) in f64, src/convert/manifest.ts:75-118; f16
manifests cast every tensor once, src/convert/manifest.ts:197-210).

Inputs follow the BASELINE configurations: token ids uniform in the stated ranges between the
family's special tokens, ragged lengths from a lognormal for the ModernBERT and cross-encoder
throughput runs. All draws come from numpy default_rng(seed).
"""
from __future__ import annotations

import math

import numpy as np

from .spec import manifest_tensor_shapes, spec_from_hf_config, tensor_names_for

# HF config.json stand-ins of the five BASELINE configurations (plus extras the reference reads
# beside the config: task, tokenizer template, sentence-transformers modules).
CONFIGS: dict[str, dict] = {
    # C1: MiniLM-L6 BERT embedding encoder, f32 (the reference's CPU-runnable case)
    "minilm-l6": {
        "config": {"model_type": "bert", "hidden_size": 384, "num_hidden_layers": 6, "num_attention_heads": 12,
                   "intermediate_size": 1536, "hidden_act": "gelu", "vocab_size": 30522,
                   "max_position_embeddings": 512, "type_vocab_size": 2, "layer_norm_eps": 1e-12},
        "extras": {"task": "embeddings",
                   "sentenceTransformers": {"pooling": {"pooling_mode_mean_tokens": True}, "normalize": True}},
        "f16": False, "special": (101, 102), "ids": (1000, 30521),
    },
    # C2: RoBERTa-base 3-label classifier, f16
    "roberta-base": {
        "config": {"model_type": "roberta", "hidden_size": 768, "num_hidden_layers": 12, "num_attention_heads": 12,
                   "intermediate_size": 3072, "hidden_act": "gelu", "vocab_size": 50265,
                   "max_position_embeddings": 514, "type_vocab_size": 1, "layer_norm_eps": 1e-5,
                   "pad_token_id": 1, "num_labels": 3},
        "extras": {"task": "sequence-classification", "template": [0, None, 2]},
        "f16": True, "special": (0, 2), "ids": (4, 50264),
    },
    # C3: DeBERTa-v3-base 2-label classifier, disentangled c2p + p2c attention, f16
    "deberta-v3-base": {
        "config": {"model_type": "deberta-v2", "hidden_size": 768, "num_hidden_layers": 12,
                   "num_attention_heads": 12, "intermediate_size": 3072, "hidden_act": "gelu",
                   "vocab_size": 128100, "max_position_embeddings": 512, "type_vocab_size": 0,
                   "layer_norm_eps": 1e-7, "relative_attention": True, "position_buckets": 256,
                   "max_relative_positions": -1, "pos_att_type": ["p2c", "c2p"], "share_att_key": True,
                   "norm_rel_ebd": "layer_norm", "position_biased_input": False, "num_labels": 2,
                   "pooler_hidden_size": 768, "pooler_hidden_act": "gelu"},
        "extras": {"task": "sequence-classification"},
        "f16": True, "special": (1, 2), "ids": (3, 128099),
    },
    # C4: ModernBERT-base embedding encoder, f16
    "modernbert-base": {
        "config": {"model_type": "modernbert", "hidden_size": 768, "num_hidden_layers": 22,
                   "num_attention_heads": 12, "intermediate_size": 1152, "vocab_size": 50368,
                   "max_position_embeddings": 8192, "norm_eps": 1e-5, "norm_bias": False,
                   "attention_bias": False, "mlp_bias": False, "global_attn_every_n_layers": 3,
                   "local_attention": 128, "global_rope_theta": 160000.0, "local_rope_theta": 10000.0},
        "extras": {"task": "embeddings",
                   "sentenceTransformers": {"pooling": {"pooling_mode_mean_tokens": True}, "normalize": True}},
        "f16": True, "special": (50281, 50282), "ids": (5, 50279),
    },
    # C5: multilingual MiniLM-L12 cross-encoder (XLM-R shape), 1-logit rerank head, f16
    "mminilm-l12-xlmr": {
        "config": {"model_type": "xlm-roberta", "hidden_size": 384, "num_hidden_layers": 12,
                   "num_attention_heads": 12, "intermediate_size": 1536, "hidden_act": "gelu",
                   "vocab_size": 250002, "max_position_embeddings": 514, "type_vocab_size": 1,
                   "layer_norm_eps": 1e-5, "pad_token_id": 1, "num_labels": 1},
        "extras": {"task": "reranking", "template": [0, None, 2]},
        "f16": True, "special": (0, 2), "ids": (4, 250001),
    },
}


def model(name: str, **overrides) -> tuple[dict, dict]:
    """(spec, head) of a named configuration; overrides replace HF config keys (tests use small
    layer counts and vocabularies)."""
    c = CONFIGS[name]
    cfg = {**c["config"], **overrides}
    spec, head, _ = spec_from_hf_config(cfg, c["extras"])
    return spec, head


def _layer_norm64(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float) -> np.ndarray:
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return (x - mean) / np.sqrt(var + eps) * w + b


def random_weights(spec: dict, head: dict, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """f32 tensors of a converted random-init model, name -> array (canonical names of
    src/plan/spec.ts:109-183)."""
    rng = np.random.default_rng(seed)
    shapes = manifest_tensor_shapes(spec, head)
    out: dict[str, np.ndarray] = {}
    for name, shape in shapes.items():
        if name.endswith(("pos_key", "pos_query")):
            continue
        leaf = name.rsplit(".", 1)[-1]
        is_norm_w = leaf == "weight" and len(shape) == 1
        a = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        if is_norm_w:
            a += np.float32(1.0)
        out[name] = a
    if spec["attention"]["kind"] == "deberta-relative":
        # src/convert/manifest.ts:75-118: pos = LayerNorm(rel_embeddings) W^T + b in f64, with the
        # key projection for pos_key and the query projection for pos_query (share_att_key).
        H = spec["hidden"]
        rows = 2 * spec["attention"]["rel"]["buckets"]
        rel = rng.standard_normal((rows, H)).astype(np.float32) * np.float32(std)
        g = (1 + rng.standard_normal(H) * std).astype(np.float32)
        bta = (rng.standard_normal(H) * std).astype(np.float32)
        ln = _layer_norm64(rel.astype(np.float64), g.astype(np.float64), bta.astype(np.float64),
                           spec["block"]["norm"]["eps"])
        names = tensor_names_for(spec["family"], spec)
        for l in range(spec["layers"]):
            t = names.layer(l)
            w = out[t["qkvW"]].astype(np.float64)
            b = out[t["qkvB"]].astype(np.float64)
            wq, wk = w[:H], w[H:2 * H]
            bq, bk = b[:H], b[H:2 * H]
            out[t["posKey"]] = (ln @ wk.T + bk).astype(np.float32)
            out[t["posQuery"]] = (ln @ wq.T + bq).astype(np.float32)
    return out


def to_f16(tensors: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """The f16 manifest: every tensor cast once; values outside the f16 range are an error
    (src/convert/manifest.ts:197-210)."""
    out = {}
    for k, v in tensors.items():
        h = v.astype(np.float16)
        if not np.all(np.isfinite(h)):
            raise ValueError(f"{k}: value outside the f16 range")
        out[k] = h
    return out


def seq_lengths(name: str, n: int, seed: int, max_len: int = 512) -> np.ndarray:
    """Token counts (specials included) of n synthetic inputs of a configuration."""
    rng = np.random.default_rng(seed)
    if name == "modernbert-base":
        # lognormal, median 45, sigma 0.8, clipped to [8, 512]
        return np.clip(np.round(rng.lognormal(math.log(45), 0.8, n)), 8, min(512, max_len)).astype(np.int32)
    if name == "mminilm-l12-xlmr":
        # query U[4, 32], passage lognormal median 90 (sigma 0.8), <s> q </s></s> p </s> <= 512
        q = rng.integers(4, 33, n)
        p = np.round(rng.lognormal(math.log(90), 0.8, n)).astype(np.int64)
        p = np.clip(p, 1, min(512, max_len) - 4 - q)
        return (q + p + 4).astype(np.int32)
    raise ValueError(f"{name} has fixed-length inputs")


def token_ids(name: str, lengths, seed: int) -> list[np.ndarray]:
    """Token ids per input: the family's leading and trailing special tokens around ids drawn
    uniformly from the configuration's range (cross-encoder pairs carry the </s></s> joint)."""
    c = CONFIGS[name]
    lo, hi = c["ids"]
    first, last = c["special"]
    rng = np.random.default_rng(seed)
    out = []
    for n in lengths:
        ids = rng.integers(lo, hi + 1, int(n)).astype(np.int64)
        ids[0] = first
        ids[-1] = last
        if name == "mminilm-l12-xlmr" and n >= 6:
            j = max(2, min(int(n) - 3, 2 + int(rng.integers(4, 33))))
            ids[j] = last
            ids[j + 1] = last
        out.append(ids)
    return out

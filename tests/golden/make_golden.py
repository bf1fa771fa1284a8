"""Generates tests/golden/forward_golden.json: expected encoder outputs of tiny random-init
models of every family, computed by the reference's own f64 executable specification
``convert/k28_forward.py`` (``encoder`` + ``head_forward``, convert/k28_forward.py:148-264)
imported from the reference checkout. Run in the build container, where the reference exists:

    python tests/golden/make_golden.py <path to the reference checkout>

The weights are not stored: they are regenerated from the recorded seed by
kleinhirn_b200.synthetic.random_weights, and the file records the sha256 of the generated
bytes so a change of the generator fails the tests instead of comparing against other weights.
The tests read the JSON only; they never import the reference.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from kleinhirn_b200.spec import spec_from_hf_config  # noqa: E402
from kleinhirn_b200.synthetic import random_weights  # noqa: E402

# Tiny members of the families and head variants: hidden 64, 2 heads (D 32), 1-3 layers,
# vocabulary 96.
CASES = [
    {"name": "bert-embed-mean", "seed": 11,
     "config": {"model_type": "bert", "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 80,
                "type_vocab_size": 2, "layer_norm_eps": 1e-12},
     "extras": {"task": "embeddings", "sentenceTransformers": {"pooling": {"pooling_mode_mean_tokens": True},
                                                               "normalize": True}},
     "lengths": [5, 13, 32]},
    {"name": "roberta-classify", "seed": 12,
     "config": {"model_type": "roberta", "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 82,
                "type_vocab_size": 1, "layer_norm_eps": 1e-5, "pad_token_id": 1, "num_labels": 3},
     "extras": {"task": "sequence-classification", "template": [0, None, 2]},
     "lengths": [6, 17, 31]},
    {"name": "xlmr-rerank", "seed": 13,
     "config": {"model_type": "xlm-roberta", "hidden_size": 64, "num_hidden_layers": 1, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 82,
                "type_vocab_size": 1, "layer_norm_eps": 1e-5, "pad_token_id": 1, "num_labels": 1},
     "extras": {"task": "reranking", "template": [0, None, 2]},
     "lengths": [4, 29]},
    {"name": "distilbert-classify", "seed": 14,
     "config": {"model_type": "distilbert", "dim": 64, "n_layers": 2, "n_heads": 2, "hidden_dim": 128,
                "activation": "gelu", "vocab_size": 96, "max_position_embeddings": 80, "num_labels": 2},
     "extras": {"task": "sequence-classification"},
     "lengths": [7, 20]},
    {"name": "deberta-v3-classify", "seed": 15,
     "config": {"model_type": "deberta-v2", "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 64,
                "type_vocab_size": 0, "layer_norm_eps": 1e-7, "relative_attention": True, "position_buckets": 16,
                "max_relative_positions": -1, "pos_att_type": ["p2c", "c2p"], "share_att_key": True,
                "norm_rel_ebd": "layer_norm", "position_biased_input": False, "num_labels": 2,
                "pooler_hidden_size": 64, "pooler_hidden_act": "gelu"},
     "extras": {"task": "sequence-classification"},
     "lengths": [9, 32]},
    {"name": "modernbert-embed", "seed": 16,
     "config": {"model_type": "modernbert", "hidden_size": 64, "num_hidden_layers": 3, "num_attention_heads": 2,
                "intermediate_size": 96, "vocab_size": 96, "max_position_embeddings": 128, "norm_eps": 1e-5,
                "norm_bias": False, "attention_bias": False, "mlp_bias": False, "global_attn_every_n_layers": 3,
                "local_attention": 8, "global_rope_theta": 160000.0, "local_rope_theta": 10000.0},
     "extras": {"task": "embeddings", "sentenceTransformers": {"pooling": {"pooling_mode_mean_tokens": True},
                                                               "normalize": True}},
     "lengths": [6, 19, 32]},
    # ELECTRA: embeddings of width 32 projected to the hidden width (src/plan/build.ts:166-169)
    {"name": "electra-classify", "seed": 17,
     "config": {"model_type": "electra", "hidden_size": 64, "embedding_size": 32, "num_hidden_layers": 2,
                "num_attention_heads": 2, "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96,
                "max_position_embeddings": 80, "type_vocab_size": 2, "layer_norm_eps": 1e-12, "num_labels": 2},
     "extras": {"task": "sequence-classification"},
     "lengths": [5, 23]},
    # DeBERTa-v2 with the convolution after layer 0 (im2col + conv GEMM, src/plan/build.ts:196-210)
    {"name": "deberta-v2-conv-classify", "seed": 18,
     "config": {"model_type": "deberta-v2", "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 64,
                "type_vocab_size": 0, "layer_norm_eps": 1e-7, "relative_attention": True, "position_buckets": 16,
                "max_relative_positions": -1, "pos_att_type": ["p2c", "c2p"], "share_att_key": True,
                "norm_rel_ebd": "layer_norm", "position_biased_input": False, "num_labels": 3,
                "conv_kernel_size": 3, "conv_act": "tanh",
                "pooler_hidden_size": 64, "pooler_hidden_act": "gelu"},
     "extras": {"task": "sequence-classification"},
     "lengths": [8, 30]},
    # token classification: one logit row per token (src/plan/build.ts:296-357)
    {"name": "bert-token", "seed": 19,
     "config": {"model_type": "bert", "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 80,
                "type_vocab_size": 2, "layer_norm_eps": 1e-12, "num_labels": 5},
     "extras": {"task": "token-classification"},
     "lengths": [7, 26]},
    # max and CLS pooling of embedding heads
    {"name": "bert-embed-max", "seed": 20,
     "config": {"model_type": "bert", "hidden_size": 64, "num_hidden_layers": 1, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 80,
                "type_vocab_size": 2, "layer_norm_eps": 1e-12},
     "extras": {"task": "embeddings", "sentenceTransformers": {"pooling": {"pooling_mode_max_tokens": True},
                                                               "normalize": True}},
     "lengths": [4, 21]},
    {"name": "bert-embed-cls", "seed": 21,
     "config": {"model_type": "bert", "hidden_size": 64, "num_hidden_layers": 1, "num_attention_heads": 2,
                "intermediate_size": 128, "hidden_act": "gelu", "vocab_size": 96, "max_position_embeddings": 80,
                "type_vocab_size": 2, "layer_norm_eps": 1e-12},
     "extras": {"task": "embeddings", "sentenceTransformers": {"pooling": {"pooling_mode_cls_token": True},
                                                               "normalize": True}},
     "lengths": [3, 27]},
]


def weights_digest(tensors: dict[str, np.ndarray]) -> str:
    h = hashlib.sha256()
    for k in sorted(tensors):
        h.update(k.encode())
        h.update(np.ascontiguousarray(tensors[k], dtype=np.float32).tobytes())
    return h.hexdigest()


def main(ref: Path) -> None:
    sys.path.insert(0, str(ref / "convert"))
    import k28_forward as kf  # the reference's executable specification

    rng = np.random.default_rng(2024)
    out = {"source": "convert/k28_forward.py (encoder, head_forward), float64", "cases": []}
    for case in CASES:
        spec, head, _ = spec_from_hf_config(case["config"], case["extras"])
        w = random_weights(spec, head, seed=case["seed"])
        T = {k: v.astype(np.float64) for k, v in w.items()}
        items = []
        for n in case["lengths"]:
            ids = rng.integers(3, spec["vocab"], n)
            ids[0], ids[-1] = 0 if spec["family"] in ("roberta", "xlm-roberta") else 2, 2
            tt = np.zeros(n, dtype=np.int64)
            x = kf.encoder(T, spec, ids, tt)
            r = kf.head_forward(T, head, x)
            if head["type"] == "embed":
                pooled, final = r
                want = pooled  # the plan outputs the pooled row; L2 runs in JS (src/tasks.ts:35-45)
            else:
                want = r
            items.append({"ids": [int(i) for i in ids], "want": [float(v) for v in np.ravel(want)]})
        out["cases"].append({"name": case["name"], "seed": case["seed"], "config": case["config"],
                             "extras": case["extras"], "weights_sha256": weights_digest(w), "items": items})
    path = Path(__file__).resolve().parent / "forward_golden.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the reference checkout>")
    main(Path(sys.argv[1]))

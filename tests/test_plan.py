"""Plan builder restatement (src/plan/build.ts, layers.ts, spec.ts, hf.ts) and host packing
(src/encoder.ts:273-314): structure, index tables and bit-exact packing."""
import math

import numpy as np
import pytest

from kleinhirn_b200 import synthetic
from kleinhirn_b200.encoder import mask_and_types, packed_inputs, word_rows, next_batch_size, batch_stride
from kleinhirn_b200.plan import build_plan, plan_ops, plan_to_json, rel_bucket_index, rel_pos_table, rope_table
from kleinhirn_b200.spec import position_rows, spec_from_hf_config


def kernels(plan):
    return [o["kernel"] for o in plan_ops(plan)]


def test_post_norm_layer_ops_bert():
    spec, head = synthetic.model("minilm-l6")
    plan = build_plan(spec, head, 128, 1, 0, False)
    ks = kernels(plan)
    assert ks[0] == "embln"
    # one layer: qkv, attS, attP, attV, attnOut, lnA, ffn1, ffn2, lnF (src/plan/layers.ts:118-149)
    assert ks[1:10] == ["mmtile", "attscore", "attsoftmax", "attpv", "mmtile", "layernorm", "mmtile", "mmtile",
                        "layernorm"]
    assert ks[-1] == "pool"
    assert plan["output"]["rows"] == 1 and plan["output"]["cols"] == 384


def test_pre_norm_layer_ops_modernbert_and_windows():
    spec, head = synthetic.model("modernbert-base", num_hidden_layers=4)
    plan = build_plan(spec, head, 512, 1, 0, True)
    segs = {s["name"]: s for s in plan["segments"]}
    l0 = [o["kernel"] for o in segs["layer0"]["ops"]]
    assert l0[0] == "mmtile" and "layernorm" == l0[l0.index("add") + 1]  # identity first norm in layer 0
    l1 = [o["kernel"] for o in segs["layer1"]["ops"]]
    assert l1[:3] == ["layernorm", "mmtile", "rope"]
    win = {s["name"]: next(o for o in s["ops"] if o["kernel"] == "attsoftmax")["constants"]["WINDOW"]
           for s in plan["segments"] if s["name"].startswith("layer")}
    assert win == {"layer0": 0, "layer1": 64, "layer2": 64, "layer3": 0}
    rope_tables = {next(o for o in s["ops"] if o["kernel"] == "rope")["bind"][1]
                   for s in plan["segments"] if s["name"].startswith("layer")}
    assert rope_tables == {"cossinG", "cossinL"}


def test_deberta_relative_plan_constants():
    spec, head = synthetic.model("deberta-v3-base", num_hidden_layers=1)
    plan = build_plan(spec, head, 512, 1, 0, True)
    ops = plan_ops(plan)
    rel = [o for o in ops if o["kernel"] == "attrel"]
    assert [o["constants"]["PART"] for o in rel] == [0, 1]
    assert rel[0]["constants"]["MOFF"] == 1 and rel[0]["constants"]["NM"] == 511
    soft = next(o for o in ops if o["kernel"] == "attsoftrel")
    assert soft["constants"]["INVSCALE"] == pytest.approx(1 / math.sqrt(3 * 64))
    assert kernels(plan)[0] == "layernorm" and ops[0]["constants"]["MODE"] == 1


def test_rel_bucket_table_properties():
    t = rel_pos_table(512, 256, 512).reshape(512, 512).astype(np.int64)
    assert t[0, 0] == 256 and t.min() >= 0 and t.max() <= 511
    # monotone in i - j (the property the reachable-window skipping relies on)
    for i in (0, 100, 511):
        assert np.all(np.diff(t[i, ::-1]) >= 0)
    assert rel_bucket_index(0, 511, 256, 512) == 1 and rel_bucket_index(511, 0, 256, 512) == 511


def test_rope_table():
    t = rope_table(8, 10000.0, 6).reshape(8, 12)
    f = 3 * 10000 ** (-(2 * 1) / 6)
    assert t[3, 1] == np.float32(math.cos(f)) and t[3, 7] == np.float32(math.sin(f))


def test_position_rows_and_packing():
    assert position_rows(1, [0, 5, 1, 7]) == [2, 3, 1, 4]
    spec, head = synthetic.model("roberta-base", num_hidden_layers=1)
    inputs = [{"inputIds": [0, 10, 11, 2]}, {"inputIds": [0, 9, 2]}]
    mask, types = mask_and_types(spec, inputs, 8)
    assert mask.tolist() == [1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 0, 0, 0, 0, 0]
    assert (types >> 16).tolist() == [2, 3, 4, 5, 1, 1, 1, 1, 2, 3, 4, 1, 1, 1, 1, 1]
    table = np.arange(50265 * 2, dtype=np.float32).reshape(-1, 2)[:, :2]
    emb, ptypes, lens = packed_inputs(spec, table, [np.array(x["inputIds"]) for x in inputs])
    assert lens.tolist() == [4, 3]
    # the ragged packing equals the B = 1 packing of each sequence, bit for bit
    assert ptypes.tolist() == types[:4].tolist() + types[8:11].tolist()
    wr = word_rows(table, inputs, 8)
    assert np.array_equal(emb, np.concatenate([wr[:4], wr[8:11]]))


def test_batch_helpers():
    assert [next_batch_size(n) for n in (1, 2, 5, 16)] == [1, 4, 8, 16]
    assert batch_stride(65) == 128 and batch_stride(64) == 64


def test_plan_json_roundtrip_and_init():
    import base64, json
    spec, head = synthetic.model("deberta-v3-base", num_hidden_layers=1)
    plan = build_plan(spec, head, 64, 1, 0, True)
    js = json.loads(plan_to_json(plan))
    rel = next(b for b in js["buffers"] if b["id"] == "relidx")
    table = np.frombuffer(base64.b64decode(rel["init_b64"]), dtype=np.uint32)
    assert np.array_equal(table, rel_pos_table(64, 256, 512))


def test_config_errors_name_the_key():
    with pytest.raises(ValueError, match="model_type"):
        spec_from_hf_config({"model_type": "gpt2"}, {"task": "embeddings"})
    cfg = dict(synthetic.CONFIGS["deberta-v3-base"]["config"], share_att_key=False)
    with pytest.raises(ValueError, match="share_att_key"):
        spec_from_hf_config(cfg, {"task": "sequence-classification"})


def test_missing_library_fails_loudly(tmp_path):
    from kleinhirn_b200.backend import load_library
    with pytest.raises(FileNotFoundError):
        load_library(tmp_path / "libkhcuda.so")

"""Plan-mode runs replayed as CUDA graphs (kh_run: eager on the first run with a row count,
captured on the second, replayed after) give the same outputs as eager runs, bit for bit: the
same kernels on the same inputs. Row counts alternate so that several graphs of one plan are
live, and new inputs are uploaded between replays (the graph reads the plan's buffers, not a
copy). Reference behaviour: PlanRunner.upload / run / readOutput (src/backend.ts:14-28)."""
import os

import numpy as np
import pytest

from harness import Model
from kleinhirn_b200 import synthetic
from kleinhirn_b200.encoder import mask_and_types, word_rows
from kleinhirn_b200.plan import build_plan

pytestmark = pytest.mark.gpu


def run_all(m, id_lists, length, eager):
    from kleinhirn_b200.backend import CudaBackend
    old = os.environ.pop("KH_NO_GRAPHS", None)
    if eager:
        os.environ["KH_NO_GRAPHS"] = "1"
    try:
        be = CudaBackend(m.weights)
        r = be.runner(build_plan(m.spec, m.head, length, 1, 0, m.f16))
    finally:
        os.environ.pop("KH_NO_GRAPHS", None)
        if old is not None:
            os.environ["KH_NO_GRAPHS"] = old
    outs = []
    for ids in id_lists:
        inputs = [{"inputIds": list(ids)}]
        mask, types = mask_and_types(m.spec, inputs, length)
        r.upload(word_rows(m.word_table, inputs, length), mask, types)
        r.run(len(ids))
        outs.append(r.read_output().copy())
    r.destroy()
    be.dispose()
    return outs


@pytest.mark.parametrize("name", ["minilm-l6", "mminilm-l12-xlmr", "deberta-v3-base"])
def test_graph_replays_equal_eager_runs(name):
    cfg = dict(synthetic.CONFIGS[name]["config"])
    cfg["num_hidden_layers"] = 2
    cfg["vocab_size"] = 512
    m = Model(cfg, synthetic.CONFIGS[name]["extras"], seed=3, f16=synthetic.CONFIGS[name]["f16"])
    lengths = [9, 17, 9, 17, 9, 30, 17, 9, 30, 30]
    ids = [np.minimum(x, 511) for x in synthetic.token_ids(name, lengths, 5)]
    length = 128
    graphed = run_all(m, ids, length, eager=False)
    eager = run_all(m, ids, length, eager=True)
    for n, g, e in zip(lengths, graphed, eager):
        assert np.array_equal(g, e), f"{name} rows {n}: max diff {np.abs(g - e).max()}"


def run_bulk_all(m, batches, length, chunk, eager):
    from kleinhirn_b200.backend import CudaBackend
    from kleinhirn_b200.encoder import packed_inputs
    old = os.environ.pop("KH_NO_GRAPHS", None)
    if eager:
        os.environ["KH_NO_GRAPHS"] = "1"
    try:
        be = CudaBackend(m.weights)
        r = be.runner(build_plan(m.spec, m.head, length, 1, 0, m.f16))
        tokens = max(sum(len(x) for x in ids) for ids in batches)
        b = be.bulk(r, tokens, max(len(ids) for ids in batches), chunk)
    finally:
        os.environ.pop("KH_NO_GRAPHS", None)
        if old is not None:
            os.environ["KH_NO_GRAPHS"] = old
    outs = []
    for ids in batches:
        emb, types, lens = packed_inputs(m.spec, m.word_table, [np.asarray(x) for x in ids])
        outs.append(np.array(b.run_batch(lens, emb, types if "typeIds" in r.plan["inputs"] else None), copy=True))
    b.close()
    r.destroy()
    be.dispose()
    return outs


@pytest.mark.parametrize("name", ["minilm-l6", "mminilm-l12-xlmr"])
def test_bulk_graph_replays_equal_eager_runs(name):
    """Bulk runs whose chunks repeat the previous run's shapes (the same lengths, new ids) replay a
    graph from the second repeat on; other shapes run eagerly. Outputs equal eager runs bit for bit."""
    cfg = dict(synthetic.CONFIGS[name]["config"])
    cfg["num_hidden_layers"] = 2
    cfg["vocab_size"] = 512
    m = Model(cfg, synthetic.CONFIGS[name]["extras"], seed=3, f16=synthetic.CONFIGS[name]["f16"])
    la, lb = [9, 30, 17, 64, 5], [40, 12, 33]
    batches = []
    for k, lens in enumerate([la, la, la, lb, la, la]):
        batches.append([np.minimum(x, 511) for x in synthetic.token_ids(name, lens, 11 + k)])
    graphed = run_bulk_all(m, batches, 128, 96, eager=False)
    eager = run_bulk_all(m, batches, 128, 96, eager=True)
    for k, (g, e) in enumerate(zip(graphed, eager)):
        assert np.array_equal(g, e), f"{name} batch {k}: max diff {np.abs(g - e).max()}"

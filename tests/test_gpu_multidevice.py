"""Several devices from one process: one context per device (kh_init), each driven by its own
host thread, as a single host process (the Node addon) would spread a batch over the GPUs of a
node. The kernels' per-device settings (shared-memory limits) are made once per device, so every
context computes what a context alone computes. Needs two GPUs; skipped otherwise."""
import threading

import numpy as np
import pytest

from harness import Model, cuda_forward_bulk
from kleinhirn_b200 import synthetic

pytestmark = pytest.mark.gpu


def _devices() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_devices() < 2, reason="needs two GPUs")
def test_contexts_on_two_devices_from_two_threads():
    from kleinhirn_b200.backend import CudaBackend
    name = "mminilm-l12-xlmr"
    cfg = dict(synthetic.CONFIGS[name]["config"], num_hidden_layers=2)
    m = Model(cfg, synthetic.CONFIGS[name]["extras"], seed=3, f16=True)
    lens = synthetic.seq_lengths(name, 600, 3)
    ids = [np.minimum(x, 511) for x in synthetic.token_ids(name, lens, 3)]
    halves = [ids[0::2], ids[1::2]]
    # each half alone on device 0: the reference results
    alone = []
    for h in halves:
        be0 = CudaBackend(m.weights, device=0)
        alone.append(cuda_forward_bulk(be0, m, h, 512, chunk_tokens=20000))
        be0.dispose()
    got: list = [None, None]
    errors: list = []

    def work(dev: int):
        try:
            be = CudaBackend(m.weights, device=dev)
            got[dev] = cuda_forward_bulk(be, m, halves[dev], 512, chunk_tokens=20000)
            be.dispose()
        except Exception as e:  # reported below, on the test's thread
            errors.append(e)

    threads = [threading.Thread(target=work, args=(d,)) for d in (0, 1)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for d in (0, 1):
        assert np.allclose(got[d], alone[d], rtol=2e-3, atol=2e-3), np.abs(got[d] - alone[d]).max()

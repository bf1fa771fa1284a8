"""Failure handling of a context on a live device, made in the forms that leave the GPU usable:

- a CUDA failure injected on the host (kh_inject_cuda_error) is reported by the next latching call
  and latched: every later call of the context fails with KH_ERR_STATE and the first message, as
  failIfBroken does (src/device.ts:68-81); a new context on the device works;
- a bounded device wait that nothing completes (kh_selftest_wait_limit: one CTA waits on an
  mbarrier nothing arrives on, with a 2 ms limit, no copy or MMA in flight) gives up, the call
  reports "pipeline wait timed out" and latches; the device error word is cleared by that
  report, so a new context on the device runs a forward cleanly;
- the TMA descriptor cache under concurrent host threads hands out only correct descriptors.
"""
import numpy as np
import pytest

from harness import Model, cuda_forward_plan
from test_gpu_forward import GOLDEN

pytestmark = pytest.mark.gpu

KH_ERR_CUDA, KH_ERR_STATE = 3, 4


def small_model():
    case = GOLDEN["cases"][1]
    return Model(case["config"], case["extras"], seed=case["seed"], f16=True), [it["ids"] for it in case["items"]]


def test_injected_failure_latches_and_a_new_context_works():
    from kleinhirn_b200.backend import CudaBackend, KhError
    m, ids = small_model()
    be = CudaBackend(m.weights)
    want = cuda_forward_plan(be, m, ids, 32)
    be.inject_cuda_error("cudaMemcpyAsync of the inputs")
    with pytest.raises(KhError) as first:
        cuda_forward_plan(be, m, ids, 32)
    assert first.value.status == KH_ERR_CUDA and "injected CUDA failure" in str(first.value)
    for _ in range(2):  # latched: the same message, every later call
        with pytest.raises(KhError) as later:
            cuda_forward_plan(be, m, ids, 32)
        assert later.value.status == KH_ERR_STATE
        assert "device error latched earlier" in str(later.value) and "cudaMemcpyAsync of the inputs" in str(later.value)
    assert "injected CUDA failure" in be.info()["broken"]
    be.dispose()
    fresh = CudaBackend(m.weights)
    assert np.array_equal(cuda_forward_plan(fresh, m, ids, 32), want)
    fresh.dispose()


def test_bounded_wait_gives_up_reports_and_latches():
    from kleinhirn_b200.backend import CudaBackend, KhError
    m, ids = small_model()
    be = CudaBackend(m.weights)
    want = cuda_forward_plan(be, m, ids, 32)
    with pytest.raises(KhError) as e:
        be.selftest_wait_limit(2000)
    assert e.value.status == KH_ERR_CUDA and "pipeline wait timed out" in str(e.value)
    assert "attention code 90" in str(e.value)
    with pytest.raises(KhError) as later:
        cuda_forward_plan(be, m, ids, 32)
    assert later.value.status == KH_ERR_STATE and "pipeline wait timed out" in str(later.value)
    be.dispose()
    # the report cleared the device's error word: a new context is not blamed for it
    fresh = CudaBackend(m.weights)
    assert np.array_equal(cuda_forward_plan(fresh, m, ids, 32), want)
    fresh.dispose()


def test_descriptor_cache_under_concurrent_threads():
    from kleinhirn_b200.backend import selftest_tensor_maps
    assert selftest_tensor_maps(8, 3000) == 0


def test_dispose_frees_open_plans_and_bulk_handles():
    """Backend.dispose with a plan and a bulk handle still open (an exception skipped their
    destroy): the context frees them, and their later destroy or garbage collection is a no-op."""
    import gc

    from kleinhirn_b200.backend import CudaBackend
    from kleinhirn_b200.plan import build_plan
    m, ids = small_model()
    be = CudaBackend(m.weights)
    r = be.runner(build_plan(m.spec, m.head, 32, 1, 0, True))
    b = be.bulk(r, 64, 4, 64)
    r2 = be.runner(build_plan(m.spec, m.head, 32, 1, 0, True))
    be.dispose()
    assert r.handle is None and b.handle is None and r2.handle is None
    r.destroy()
    b.close()
    del r, b, r2
    gc.collect()
    fresh = CudaBackend(m.weights)
    assert len(cuda_forward_plan(fresh, m, ids, 32)) == len(ids)
    fresh.dispose()

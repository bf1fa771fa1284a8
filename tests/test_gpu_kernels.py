"""Every per-op known-answer case of the reference (tests/wasm_plan.test.ts, ported in
kat_cases.py) through the CUDA backend's C ABI, f32 plans, against the same float64
expectations and tolerance (2e-5 relative to scale) the reference's executor meets."""
import numpy as np
import pytest

from kat_cases import all_cases, check_case

pytestmark = pytest.mark.gpu

CASES = all_cases(with_masklogits=False)


def run_on_cuda(case):
    from kleinhirn_b200.backend import CudaBackend
    be = CudaBackend()
    for name, (arr, _panel) in case.weights.items():
        be.add_tensor(name, np.ascontiguousarray(arr, dtype=np.float32))
    r = be.runner(case.plan)
    for bid, data in case.writes.items():
        r.write_buffer(bid, np.ascontiguousarray(data))
    r.run(case.rows)
    raw = r.read_buffer(case.read, 4 * case.read_count)
    out = raw.view(np.float32).copy()
    labels = [s["label"] for s in r.launches()]
    r.destroy()
    be.dispose()
    return out, labels


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_cuda_op_against_reference_f64(case):
    got, labels = run_on_cuda(case)
    check_case(case, got)
    if any(k in ("attscore", "attrel", "mbflash", "mbattention", "attention") for k in case.kernels):
        assert labels.count("attention") == 1, labels  # the group runs as one attention launch

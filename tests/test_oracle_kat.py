"""The oracle (C++ restatement of the reference's WASM executor) against the float64
expectations of the reference's per-op tests (tests/wasm_plan.test.ts), serial and threaded."""
import numpy as np
import pytest

from kat_cases import all_cases, check_case
from oracle import host

CASES = all_cases()


def run_on_oracle(case, threads=1):
    rt = host.Runtime(threads=threads, split={"rb": 4, "cb": 16, "qb": 2, "minWork": 1})
    try:
        for name, (arr, panel) in case.weights.items():
            rt.add_weight(name, list(arr.shape), arr, panel)
        p = rt.plan(case.plan)
        for bid, data in case.writes.items():
            raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
            p.buf_view(bid)[: raw.size] = raw
        p.run(case.rows)
        return p.view(case.read)[: case.read_count].copy()
    finally:
        rt.close()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_against_reference_f64(case):
    check_case(case, run_on_oracle(case))


@pytest.mark.parametrize("case", [c for c in CASES if c.kernels[0] in ("mmtile", "layernorm", "geglu", "mbflash",
                                                                         "mbattention", "attention")],
                         ids=lambda c: c.name)
def test_threads_give_the_serial_bits(case):
    """src/wasm/plan.ts:949-950: every output element is computed by one thread with the same code
    and k order, so the threaded executor gives the serial bits."""
    a = run_on_oracle(case, threads=1)
    b = run_on_oracle(case, threads=4)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32)) or np.array_equal(a, b, equal_nan=True)


def test_vexp_and_gelu_helpers():
    lib = host.lib()
    xs = np.linspace(-20, 20, 401, dtype=np.float32)
    ex = np.array([lib.oracle_vexp1(float(x)) for x in xs], dtype=np.float64)
    assert np.allclose(ex, np.exp(xs.astype(np.float64)), rtol=2e-7, atol=0)
    # clamps: below -87.34 the result stays near 1e-38 instead of 0 (src/wasm/plan.ts:57-60)
    assert 0 < lib.oracle_vexp1(-200.0) < 1e-37
    g1 = np.array([lib.oracle_vgelu1(float(x)) for x in xs])
    g2 = np.array([lib.oracle_gelu(float(x)) for x in xs])
    from kat_cases import gelu64
    assert np.allclose(g1, gelu64(xs), atol=2e-6)
    assert np.allclose(g2, gelu64(xs), atol=2e-6)

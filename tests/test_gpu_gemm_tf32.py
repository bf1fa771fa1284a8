"""Matmuls of f32 plans on the tensor cores (3xTF32 split, gemm_tf32.cu), through the C ABI.

The reference's WASM executor computes f32 plans in f32 (src/kernels/mmtile.wgsl:20-35 for the
arithmetic, tests/wasm_plan.test.ts:73-101 for its matmul test). A single TF32 product keeps 10
mantissa bits (relative error about 5e-4); the split recovers f32 accuracy, so every case here is
held to 1e-5 of sum |a| |w| (plus 1e-6 of |want|), a bound one-pass TF32 misses by two orders of
magnitude. Shapes cover M, N and K tails, K below one 32-wide stage, every activation, the
sequence-level (fixed-row) form and the bulk form of the launch list."""
import numpy as np
import pytest

from kat_cases import gelu64, mini

pytestmark = pytest.mark.gpu

ACT64 = [lambda v: v, lambda v: np.maximum(v, 0), gelu64, np.tanh, lambda v: v / (1 + np.exp(-v))]


def run_f32(plan, weights, writes, rows, read, count):
    from kleinhirn_b200.backend import CudaBackend
    be = CudaBackend()
    for k, v in weights.items():
        be.add_tensor(k, v)
    r = be.runner(plan)
    for k, v in writes.items():
        r.write_buffer(k, v)
    r.run(rows)
    out = r.read_buffer(read, 4 * count).view(np.float32).astype(np.float64)
    labels = r.launches()
    r.destroy()
    be.dispose()
    return out, labels


def check(got, A, W, b, act, what):
    A64, W64 = A.astype(np.float64), W.astype(np.float64)
    pre = A64 @ W64.T + (0 if b is None else b.astype(np.float64))
    want = ACT64[act](pre).reshape(-1)
    tol = 1e-5 * (np.abs(A64) @ np.abs(W64).T).reshape(-1) + 1e-6 * np.abs(want) + 1e-6
    err = np.abs(got - want)
    bad = err > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} off, worst {err.max():.3g} (tol {tol.min():.3g}+)"


@pytest.mark.parametrize("M,N,K", [(128, 1152, 384), (128, 1536, 384), (77, 40, 20), (300, 64, 1536), (5, 16, 8),
                                   (1000, 384, 1536), (257, 72, 44), (33, 100, 36)])
@pytest.mark.parametrize("act", [0, 2, 3])
def test_tf32x3_shapes(M, N, K, act):
    rng = np.random.default_rng(M * 13 + N * 3 + K + act)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    plan = mini([{"name": "mm", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": act},
                  "bind": ["a", "w:w", "w:b", "c"], "dispatch": [1, "rows32"]}],
                {"mask": M, "a": M * K, "c": M * N}, M, "c")
    got, labels = run_f32(plan, {"w": W, "b": b}, {"a": A}, M, "c", M * N)
    # one launch: the activations are split inside the tensor-core GEMM
    assert labels[0]["label"] == "gemm" and labels[0]["launches"] == 1, labels[:1]
    check(got, A, W, b, act, f"tf32x3 {M}x{N}x{K} act {act}")


@pytest.mark.parametrize("act", [1, 4])
def test_tf32x3_relu_silu(act):
    test_tf32x3_shapes(200, 384, 384, act)


def test_tf32x3_wide_range_and_zero_bias():
    """Values over many binades (the lo parts carry the bits a TF32 product drops) and no bias."""
    rng = np.random.default_rng(5)
    M, N, K = 150, 96, 256
    A = (rng.standard_normal((M, K)) * np.exp2(rng.integers(-12, 12, (M, K)))).astype(np.float32)
    W = (rng.standard_normal((N, K)) * np.exp2(rng.integers(-8, 8, (N, K)))).astype(np.float32)
    plan = mini([{"name": "mm", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": 0},
                  "bind": ["a", "w:w", "zero", "c"], "dispatch": [1, "rows32"]}],
                {"mask": M, "a": M * K, "c": M * N, "zero": np.zeros(N, dtype=np.float32)}, M, "c")
    got, _ = run_f32(plan, {"w": W}, {"a": A}, M, "c", M * N)
    check(got, A, W, None, 0, "wide range")


def test_tf32x3_sequence_level_rows():
    """A fixed-row (pooled head) matmul: M from the op, not the token count."""
    rng = np.random.default_rng(9)
    M, N, K = 7, 48, 64
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.1).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    plan = mini([{"name": "mm", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": 3},
                  "bind": ["a", "w:w", "w:b", "c"], "dispatch": [1, 1]}],
                {"mask": M, "a": M * K, "c": M * N}, M, "c")
    got, _ = run_f32(plan, {"w": W, "b": b}, {"a": A}, 1, "c", M * N)
    check(got, A, W, b, 3, "sequence-level")

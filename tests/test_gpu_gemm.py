"""The f16 GEMM of the plan's matmul ops on the tcgen05 path, through the C ABI: shapes with M, N and
K tails, every activation (src/kernels/mmtile.wgsl:20-35), and the three epilogues that fold the
following op into the GEMM (residual add, GeGLU, RoPE), each against a numpy model of the
reference's arithmetic with its f16 storage rounding (src/kernels/index.ts:1-3)."""
import math

import numpy as np
import pytest

from kat_cases import gelu64

pytestmark = pytest.mark.gpu

ACT64 = [lambda v: v, lambda v: np.maximum(v, 0), gelu64, np.tanh, lambda v: v / (1 + np.exp(-v))]


def f16plan(ops, buffers, L, out, batch=1):
    decls = []
    for bid, (count, init) in buffers.items():
        if init is None:
            decls.append({"id": bid, "bytes": 2 * count, "usage": "rw"})
        else:
            a = np.ascontiguousarray(init)
            decls.append({"id": bid, "bytes": a.nbytes, "usage": "rw", "init": a.tobytes()})
    decls.append({"id": "mask", "bytes": 4 * L * batch, "usage": "rw"})
    return {"f16": True, "length": L, "batch": batch, "markers": 0, "embeddingSize": 1, "buffers": decls,
            "segments": [{"name": "s", "prefix": "", "ops": ops}], "inputs": {"embeddings": "mask", "mask": "mask"},
            "output": {"buffer": out, "bytes": 2 * buffers[out][0], "dtype": "storage", "rows": buffers[out][0],
                       "cols": 1}, "captureSlots": 0, "captureSlotBytes": 0}


def run(plan, weights, writes, rows, read, count):
    from kleinhirn_b200.backend import CudaBackend
    be = CudaBackend()
    for k, v in weights.items():
        be.add_tensor(k, v)
    r = be.runner(plan)
    for k, v in writes.items():
        r.write_buffer(k, v)
    r.run(rows)
    out = r.read_buffer(read, 2 * count).view(np.float16).astype(np.float64)
    labels = r.launches()
    r.destroy()
    be.dispose()
    return out, labels


def f16(x):
    return np.asarray(x, dtype=np.float64).astype(np.float16).astype(np.float64)


def assert_f16_close(got, want, what):
    # f32 accumulation in another order, then one f16 rounding: within 2 f16 ulps plus a small floor
    tol = 2 * np.abs(want) * 2.0 ** -10 + 2e-3
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} off, worst {np.abs(got - want).max()}"


@pytest.mark.parametrize("M,N,K", [(1, 32, 64), (7, 384, 384), (128, 128, 64), (129, 1152, 384),
                                   (300, 768, 3072), (1000, 1536, 384), (77, 96, 40), (640, 2304, 768),
                                   (300, 1088, 256)])  # 256-wide tiles past N: one live warpgroup
@pytest.mark.parametrize("act", [0, 2, 3])
def test_gemm_shapes(M, N, K, act):
    rng = np.random.default_rng(M * 7 + N + K + act)
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float16)
    plan = f16plan([{"name": "mm", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": act},
                     "bind": ["a", "w:w", "w:b", "c"], "dispatch": [1, "rows32"]}],
                   {"a": (M * K, None), "c": (M * N, None)}, M, "c")
    got, labels = run(plan, {"w": W, "b": b}, {"a": A}, M, "c", M * N)
    want = f16(ACT64[act](A.astype(np.float64) @ W.astype(np.float64).T + b.astype(np.float64)))
    assert_f16_close(got, want.reshape(-1), f"gemm {M}x{N}x{K} act {act}")


@pytest.mark.parametrize("act", [1, 4])
def test_gemm_relu_silu(act):
    test_gemm_shapes(256, 384, 384, act)


@pytest.mark.parametrize("N", [384, 768, 1152])  # 192-, 256-wide tiles, 256 past N
def test_residual_epilogue(N):
    """matmul (attnOut) followed by add (addA): x = f16(x + f16(A W^T + b))."""
    M, K, L = 300, 384, 300
    rng = np.random.default_rng(1)
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float16)
    x = rng.standard_normal((M, N)).astype(np.float16)
    ops = [{"name": "attnOut", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": 0},
            "bind": ["ctx", "w:w", "w:b", "attnOut"], "dispatch": [1, "rows32"]},
           {"name": "addA", "kernel": "add", "constants": {"TOTAL": M * N, "N": N, "MODE": 0, "L": L},
            "bind": ["x", "attnOut"], "dispatch": [1, 1]}]
    plan = f16plan(ops, {"ctx": (M * K, None), "attnOut": (M * N, None), "x": (M * N, None)}, L, "x")
    got, labels = run(plan, {"w": W, "b": b}, {"ctx": A, "x": x}, M, "x", M * N)
    assert [s["label"] for s in labels][:1] == ["gemm"] and labels[0]["ops"] == ["attnOut", "addA"]
    want = f16(x.astype(np.float64) + f16(A.astype(np.float64) @ W.astype(np.float64).T + b))
    assert_f16_close(got, want.reshape(-1), "residual")


@pytest.mark.parametrize("I", [1152, 192])  # interleave groups of 128 and 64
def test_geglu_epilogue(I):
    """matmul (ffnIn, N = 2I) followed by geglu: gate = f16(gelu(f16(a)) * f16(b))."""
    M, K, L = 200, 768, 200
    rng = np.random.default_rng(2)
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    W = (rng.standard_normal((2 * I, K)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(2 * I) * 0.1).astype(np.float16)
    ops = [{"name": "ffnIn", "kernel": "mmtile", "constants": {"M": M, "N": 2 * I, "K": K, "ACT": 0},
            "bind": ["normed", "w:w", "w:b", "mid"], "dispatch": [1, "rows32"]},
           {"name": "geglu", "kernel": "geglu", "constants": {"I": I}, "bind": ["mid", "gate"], "dispatch": ["rows", 1]}]
    plan = f16plan(ops, {"normed": (M * K, None), "mid": (M * 2 * I, None), "gate": (M * I, None)}, L, "gate")
    got, labels = run(plan, {"w": W, "b": b}, {"normed": A}, M, "gate", M * I)
    assert labels[0]["ops"] == ["ffnIn", "geglu"]
    mid = f16(A.astype(np.float64) @ W.astype(np.float64).T + b)
    want = f16(gelu64(mid[:, :I]) * mid[:, I:])
    assert_f16_close(got, want.reshape(-1), "geglu")


@pytest.mark.parametrize("H", [12, 6])  # N = 2304 (256-wide tiles) and 1152 (128-wide)
def test_rope_epilogue(H):
    """matmul (qkv) followed by rope: q and k heads rotated with the table row of the position."""
    D = 64
    M, N, K, L = 150, 3 * H * D, 768, 150
    rng = np.random.default_rng(3)
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    table = np.zeros(L * 2 * D, dtype=np.float32)
    for i in range(L):
        for d in range(D // 2):
            f = i * 10000.0 ** (-(2 * d) / D)
            table[i * 2 * D + d] = math.cos(f)
            table[i * 2 * D + D + d] = math.sin(f)
    ops = [{"name": "qkv", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": 0},
            "bind": ["normed", "w:w", "zero", "qkv"], "dispatch": [1, "rows32"]},
           {"name": "rope", "kernel": "rope", "constants": {"L": L, "H": H, "D": D}, "bind": ["qkv", "cs"],
            "dispatch": ["rows", 2 * H]}]
    plan = f16plan(ops, {"normed": (M * K, None), "qkv": (M * N, None), "cs": (0, table),
                         "zero": (0, np.zeros(N, dtype=np.float16))}, L, "qkv")
    got, labels = run(plan, {"w": W}, {"normed": A}, M, "qkv", M * N)
    assert labels[0]["ops"] == ["qkv", "rope"]
    q = f16(A.astype(np.float64) @ W.astype(np.float64).T).reshape(M, 3 * H, D)
    t = table.reshape(L, 2 * D).astype(np.float64)
    c, s = t[:M, : D // 2][:, None, :], t[:M, D: D + D // 2][:, None, :]
    x, y = q[:, : 2 * H, : D // 2].copy(), q[:, : 2 * H, D // 2:].copy()
    q[:, : 2 * H, : D // 2] = x * c - y * s
    q[:, : 2 * H, D // 2:] = y * c + x * s
    assert_f16_close(got, f16(q).reshape(-1), "rope")


@pytest.mark.parametrize("N,K,M", [(384, 384, 300), (384, 1536, 700), (256, 768, 129)])
def test_addnorm_epilogue(N, K, M):
    """matmul followed by layernorm mode 2 over (residual, matmul output):
    out = LN(R + f16(A W^T + b)) * w + beta (two-pass variance, src/kernels/layernorm.wgsl)."""
    L = M
    eps = 1e-5
    rng = np.random.default_rng(N + K + M)
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float16)
    R = rng.standard_normal((M, N)).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(N)).astype(np.float16)
    beta = (0.1 * rng.standard_normal(N)).astype(np.float16)
    ops = [{"name": "attnOut", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": 0},
            "bind": ["ctx", "w:w", "w:b", "attnOut"], "dispatch": [1, "rows32"]},
           {"name": "lnA", "kernel": "layernorm", "constants": {"N": N, "MODE": 2, "EPS": eps},
            "bind": ["x", "attnOut", "w:g", "w:beta", "mask", "tmp"], "dispatch": ["rows", 1]}]
    plan = f16plan(ops, {"ctx": (M * K, None), "attnOut": (M * N, None), "x": (M * N, None), "tmp": (M * N, None)},
                   L, "tmp")
    got, labels = run(plan, {"w": W, "b": b, "g": g, "beta": beta}, {"ctx": A, "x": R}, M, "tmp", M * N)
    assert labels[0]["label"] == "gemm" and labels[0]["ops"] == ["attnOut", "lnA"]
    y = f16(A.astype(np.float64) @ W.astype(np.float64).T + b)
    v = R.astype(np.float64) + y
    mean = v.mean(axis=1, keepdims=True)
    var = ((v - mean) ** 2).mean(axis=1, keepdims=True)
    want = f16((v - mean) / np.sqrt(var + eps) * g.astype(np.float64) + beta.astype(np.float64))
    assert_f16_close(got, want.reshape(-1), f"add+layernorm N={N} K={K}")


# Launches of the C5 size: many 256-row blocks per CTA pair (the last one half full), the
# persistent tile loop, both accumulators and the stage ring wrapping many times.
@pytest.mark.parametrize("N,K,act", [(1152, 384, 0), (1536, 384, 2), (768, 200, 3)])
def test_gemm_row_block_schedule(N, K, act):
    from kleinhirn_b200.backend import CudaBackend
    M = 80_000  # 313 row blocks (the last one half full) against 74 pairs
    rng = np.random.default_rng(N + K)
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float16)
    plan = f16plan([{"name": "mm", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": act},
                     "bind": ["a", "w:w", "w:b", "c"], "dispatch": [1, "rows32"]}],
                   {"a": (M * K, None), "c": (M * N, None)}, M, "c")
    be = CudaBackend()
    be.add_tensor("w", W)
    be.add_tensor("b", b)
    r = be.runner(plan)
    r.write_buffer("a", A)
    r.run(M)
    C = r.read_buffer("c", 2 * M * N).view(np.float16).reshape(M, N)
    r.destroy()
    be.dispose()
    rows = np.unique(np.concatenate([rng.integers(0, M, 3000), np.arange(M - 300, M), np.arange(0, 300)]))
    want = f16(ACT64[act](A[rows].astype(np.float64) @ W.astype(np.float64).T + b.astype(np.float64)))
    assert_f16_close(C[rows].astype(np.float64).reshape(-1), want.reshape(-1), f"gemm {M}x{N}x{K} act {act}")

"""Attention of f16 plans on the tensor-core path, through the C ABI, against the float64
reference of the reference's own attention test (tests/wasm_plan.test.ts:299-333): batches of
sequences packed into shared 128-row tiles, prefix masks with NaN-poisoned padding rows (they
must never enter a sum), masked query rows exactly zero, sliding windows, head dimensions 32 and
64, sequences longer than one 128-key tile."""
import math

import numpy as np
import pytest

from kat_cases import attention_ref, prefix_mask

pytestmark = pytest.mark.gpu


def run_attention(qkv16, mask, L, B, H, D, scale, window, rows, op="mbflash"):
    from kleinhirn_b200.backend import CudaBackend
    hd = H * D
    ops = [{"name": "attn", "kernel": op, "constants": {"L": L, "H": H, "D": D, "SCALE": scale, "WINDOW": window,
                                                         "ROWS": B * L},
            "bind": ["qkv", "mask", "ctx"], "dispatch": [H, "rows"]}]
    plan = {"f16": True, "length": L, "batch": B, "markers": 0, "embeddingSize": 1,
            "buffers": [{"id": "qkv", "bytes": 2 * B * L * 3 * hd, "usage": "rw"},
                        {"id": "mask", "bytes": 4 * B * L, "usage": "rw"},
                        {"id": "ctx", "bytes": 2 * B * L * hd, "usage": "rw"}],
            "segments": [{"name": "s", "prefix": "", "ops": ops}], "inputs": {"embeddings": "mask", "mask": "mask"},
            "output": {"buffer": "ctx", "bytes": 2 * B * L * hd, "dtype": "storage", "rows": B * L * hd, "cols": 1},
            "captureSlots": 0, "captureSlotBytes": 0}
    be = CudaBackend()
    r = be.runner(plan)
    r.write_buffer("qkv", qkv16)
    r.write_buffer("mask", mask)
    r.run(rows)
    out = r.read_buffer("ctx", 2 * rows * hd).view(np.float16).astype(np.float64)
    r.destroy()
    be.dispose()
    return out


@pytest.mark.parametrize("D", [32, 64])
@pytest.mark.parametrize("L,lens,window", [
    (50, [50, 17, 33], 0),         # three sequences in one 128-row tile
    (300, [300, 129], 0),          # several key tiles, a sequence across tiles
    (200, [200, 150, 7, 61], 16),  # windowed layers
    (512, [512], 0),
    (96, [96, 1, 90, 64, 30], 5),
])
def test_packed_attention_f16(D, L, lens, window):
    B, H = len(lens), 2
    hd = H * D
    rng = np.random.default_rng(L + D + window)
    qkv = (rng.standard_normal(B * L * 3 * hd) * 1.5).astype(np.float16)
    mask = prefix_mask(L, lens)
    for r in range(B * L):
        if not mask[r]:
            qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
    rows = lens[0] if B == 1 else B * L
    scale = D ** -0.5
    want = attention_ref(qkv.astype(np.float32), mask, L, B, H, D, scale, window, rows)
    got = run_attention(qkv, mask, L, B, H, D, scale, window, rows)
    keep = np.repeat(mask[:rows] > 0, hd)
    assert np.all(got[~keep] == 0), "masked query rows must be exactly zero"
    err = np.abs(got[keep] - want[keep])
    tol = 4e-3 + 1e-2 * np.abs(want[keep])
    assert np.all(err <= tol), f"worst {err.max()} at {int(np.argmax(err - tol))}"


def test_single_call_rows_below_bucket():
    """B = 1 with rows < L: only the real rows exist; stale rows past them are never read."""
    L, H, D = 128, 12, 64
    hd = H * D
    rng = np.random.default_rng(9)
    qkv = rng.standard_normal(L * 3 * hd).astype(np.float16)
    qkv[77 * 3 * hd:] = np.nan
    mask = prefix_mask(L, [77])
    want = attention_ref(qkv.astype(np.float32), mask, L, 1, H, D, D ** -0.5, 0, 77)
    got = run_attention(qkv, mask, L, 1, H, D, D ** -0.5, 0, 77)
    assert np.allclose(got, want, atol=4e-3, rtol=1e-2), np.abs(got - want).max()


def relative_ref(qkv16, mask, L, B, H, D, scale_div, idx, pk16, pq16):
    """The relative attention of attention_ref (tests/wasm_plan.test.ts:299-376) vectorised, float64."""
    hd = H * D
    x = qkv16.astype(np.float64).reshape(B, L, 3, H, D)
    pk = pk16.astype(np.float64).reshape(-1, H, D)
    pq = pq16.astype(np.float64).reshape(-1, H, D)
    p = idx.reshape(L, L).astype(np.int64)
    m = mask.reshape(B, L) > 0.5
    out = np.zeros((B, L, H, D))
    for b in range(B):
        for h in range(H):
            q, k, v = x[b, :, 0, h], x[b, :, 1, h], x[b, :, 2, h]
            qs = np.nan_to_num(q) * m[b][:, None]
            ks = np.nan_to_num(k) * m[b][:, None]
            s = qs @ ks.T + (qs @ pk[:, h].T)[np.arange(L)[:, None], p] + (ks @ pq[:, h].T)[np.arange(L)[None, :], p]
            s = np.where(m[b][None, :], s / scale_div, -np.inf)
            e = np.exp(s - s.max(axis=1, keepdims=True))
            pr = e / e.sum(axis=1, keepdims=True)
            o = pr @ (np.nan_to_num(v) * m[b][:, None])
            out[b, :, h] = np.where(m[b][:, None], o, 0.0)
    return out.reshape(-1)[: B * L * hd]


def run_relative(qkv16, mask, L, B, H, D, scale_div, idx, pk16, pq16, rows):
    from kleinhirn_b200.backend import CudaBackend
    hd = H * D
    ops = [{"name": "attn", "kernel": "attention", "constants": {"L": L, "H": H, "D": D, "SCALE": scale_div},
            "bind": ["qkv", "w:pk", "w:pq", "ri", "mask", "ctx"], "dispatch": [H, "rows"]}]
    plan = {"f16": True, "length": L, "batch": B, "markers": 0, "embeddingSize": 1,
            "buffers": [{"id": "qkv", "bytes": 2 * B * L * 3 * hd, "usage": "rw"},
                        {"id": "mask", "bytes": 4 * B * L, "usage": "rw"},
                        {"id": "ri", "bytes": idx.nbytes, "usage": "rw", "init": idx.tobytes()},
                        {"id": "ctx", "bytes": 2 * B * L * hd, "usage": "rw"}],
            "segments": [{"name": "s", "prefix": "", "ops": ops}], "inputs": {"embeddings": "mask", "mask": "mask"},
            "output": {"buffer": "ctx", "bytes": 2 * B * L * hd, "dtype": "storage", "rows": B * L * hd, "cols": 1},
            "captureSlots": 0, "captureSlotBytes": 0}
    be = CudaBackend()
    be.add_tensor("pk", pk16)
    be.add_tensor("pq", pq16)
    r = be.runner(plan)
    r.write_buffer("qkv", qkv16)
    r.write_buffer("mask", mask)
    r.run(rows)
    labels = r.launches()
    out = r.read_buffer("ctx", 2 * rows * hd).view(np.float16).astype(np.float64)
    r.destroy()
    be.dispose()
    return out, labels


@pytest.mark.parametrize("L,lens,span", [
    (160, [160, 77, 100], 64),    # three sequences, 128 relative positions
    (300, [300, 129], 256),       # several key tiles, 512 relative positions (two table tiles)
])
def test_relative_attention_f16(L, lens, span):
    """DeBERTa's disentangled attention on the tensor cores: s_ij = (q_i.k_j + q_i.posKey[p_ij] +
    k_j.posQuery[p_ij]) / sqrt(3 D) with p_ij = relidx[i][j] (src/plan/layers.ts:61-80,
    tests/wasm_plan.test.ts:336-376), against float64; NaN-poisoned padding rows."""
    B, H, D = len(lens), 4, 64
    hd = H * D
    rng = np.random.default_rng(L + span)
    qkv = (rng.standard_normal(B * L * 3 * hd) * 1.2).astype(np.float16)
    mask = prefix_mask(L, lens)
    for r in range(B * L):
        if not mask[r]:
            qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
    idx = np.zeros(L * L, dtype=np.uint32)
    for i in range(L):
        idx[i * L:(i + 1) * L] = np.clip(i - np.arange(L) + span, 0, 2 * span - 1)
    pk = (rng.standard_normal((2 * span, hd)) * 0.8).astype(np.float16)
    pq = (rng.standard_normal((2 * span, hd)) * 0.8).astype(np.float16)
    scale_div = math.sqrt(3 * D)
    rows = B * L
    want = relative_ref(qkv, mask, L, B, H, D, scale_div, idx, pk, pq)
    got, labels = run_relative(qkv, mask, L, B, H, D, scale_div, idx, pk, pq, rows)
    keep = np.repeat(mask[:rows] > 0, hd)
    assert np.all(got[~keep] == 0), "masked query rows must be exactly zero"
    err = np.abs(got[keep] - want[keep])
    tol = 4e-3 + 1e-2 * np.abs(want[keep])
    assert np.all(err <= tol), f"worst {err.max()} at {int(np.argmax(err - tol))}"


def test_relative_attention_index_not_a_function_of_distance():
    """A relidx that does not depend on i - j alone (the plan builder's tables always do, but the
    plan format allows any): the kernel reads the L x L table itself instead of folding it into a
    row over i - j; against float64."""
    L, lens, span = 200, [200, 90], 64
    B, H, D = len(lens), 4, 64
    hd = H * D
    rng = np.random.default_rng(5)
    qkv = (rng.standard_normal(B * L * 3 * hd) * 1.2).astype(np.float16)
    mask = prefix_mask(L, lens)
    for r in range(B * L):
        if not mask[r]:
            qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
    i, j = np.meshgrid(np.arange(L), np.arange(L), indexing="ij")
    idx = ((7 * i + 3 * j) % (2 * span)).astype(np.uint32).reshape(-1)
    pk = (rng.standard_normal((2 * span, hd)) * 0.8).astype(np.float16)
    pq = (rng.standard_normal((2 * span, hd)) * 0.8).astype(np.float16)
    scale_div = math.sqrt(3 * D)
    rows = B * L
    want = relative_ref(qkv, mask, L, B, H, D, scale_div, idx, pk, pq)
    got, _ = run_relative(qkv, mask, L, B, H, D, scale_div, idx, pk, pq, rows)
    keep = np.repeat(mask[:rows] > 0, hd)
    assert np.all(got[~keep] == 0)
    err = np.abs(got[keep] - want[keep])
    assert np.all(err <= 4e-3 + 1e-2 * np.abs(want[keep])), err.max()


def standard_ref(qkv16, mask, L, B, H, D, scale, window):
    """attention_ref vectorised per (sequence, head), float64 (tests/wasm_plan.test.ts:299-333)."""
    x = qkv16.astype(np.float64).reshape(B, L, 3, H, D)
    m = mask.reshape(B, L) > 0.5
    pos = np.arange(L)
    near = np.abs(pos[:, None] - pos[None, :]) <= window if window else np.ones((L, L), dtype=bool)
    out = np.zeros((B, L, H, D))
    for b in range(B):
        keep = m[b][None, :] & near
        for h in range(H):
            q = np.nan_to_num(x[b, :, 0, h])
            k = np.nan_to_num(x[b, :, 1, h])
            v = np.nan_to_num(x[b, :, 2, h]) * m[b][:, None]
            s = np.where(keep, (q @ k.T) * scale, -np.inf)
            with np.errstate(invalid="ignore"):  # rows without a kept key: replaced by zeros below
                e = np.exp(s - s.max(axis=1, keepdims=True))
                o = (e / e.sum(axis=1, keepdims=True)) @ v
            out[b, :, h] = np.where(m[b][:, None], o, 0.0)
    return out.reshape(-1)


# Large launches spread 2, 4, 6 or 12 heads over the two softmax streams of a CTA (the C5 bulk
# path runs 12): B sequences of a 128-row bucket give B packed tiles, and the head group is the
# largest even divisor of 12 that still fills the 148 SMs.
@pytest.mark.parametrize("D", [32, 64])
@pytest.mark.parametrize("B,window", [(30, 0), (60, 0), (100, 16), (160, 0)], ids=["hg2", "hg4", "hg6-window", "hg12"])
def test_packed_attention_head_groups(D, B, window):
    L, H = 128, 12
    hd = H * D
    rng = np.random.default_rng(B + D)
    lens = rng.integers(40, L + 1, B).tolist()
    qkv = (rng.standard_normal(B * L * 3 * hd) * 1.5).astype(np.float16)
    mask = prefix_mask(L, lens)
    qkv.reshape(B * L, 3 * hd)[mask <= 0.5] = np.nan
    scale = D ** -0.5
    want = standard_ref(qkv, mask, L, B, H, D, scale, window)
    got = run_attention(qkv, mask, L, B, H, D, scale, window, B * L)
    keep = np.repeat(mask > 0, hd)
    assert np.all(got[~keep] == 0), "masked query rows must be exactly zero"
    err = np.abs(got[keep] - want[keep])
    tol = 4e-3 + 1e-2 * np.abs(want[keep])
    assert np.all(err <= tol), f"worst {err.max()} at {int(np.argmax(err - tol))}"


def test_relative_attention_head_groups():
    """DeBERTa's relative attention on a launch large enough for 4 heads per CTA (both streams)."""
    B, L, H, D, span = 160, 128, 4, 64, 64
    hd = H * D
    rng = np.random.default_rng(77)
    lens = rng.integers(30, L + 1, B).tolist()
    qkv = (rng.standard_normal(B * L * 3 * hd) * 1.2).astype(np.float16)
    mask = prefix_mask(L, lens)
    qkv.reshape(B * L, 3 * hd)[mask <= 0.5] = np.nan
    idx = np.zeros(L * L, dtype=np.uint32)
    for i in range(L):
        idx[i * L:(i + 1) * L] = np.clip(i - np.arange(L) + span, 0, 2 * span - 1)
    pk = (rng.standard_normal((2 * span, hd)) * 0.8).astype(np.float16)
    pq = (rng.standard_normal((2 * span, hd)) * 0.8).astype(np.float16)
    scale_div = math.sqrt(3 * D)
    want = relative_ref(qkv, mask, L, B, H, D, scale_div, idx, pk, pq)
    got, _ = run_relative(qkv, mask, L, B, H, D, scale_div, idx, pk, pq, B * L)
    keep = np.repeat(mask > 0, hd)
    assert np.all(got[~keep] == 0), "masked query rows must be exactly zero"
    err = np.abs(got[keep] - want[keep])
    tol = 4e-3 + 1e-2 * np.abs(want[keep])
    assert np.all(err <= tol), f"worst {err.max()} at {int(np.argmax(err - tol))}"


@pytest.mark.parametrize("D", [16, 48])
@pytest.mark.parametrize("L,lens,window", [
    (50, [50, 17, 33], 0),
    (300, [300, 129], 0),          # keys staged in several chunks (128 for D 16, 64 for D 48)
    (200, [200, 150, 7, 61], 16),
    (96, [96, 1, 90, 64, 30], 5),
])
def test_attention_other_head_dims_f16(D, L, lens, window):
    """Head dimensions the tensor-core kernel does not take run the shared-memory kernel
    (attention_smem_kernel): the same semantics, NaN padding rows never enter a sum."""
    test_packed_attention_f16(D, L, lens, window)

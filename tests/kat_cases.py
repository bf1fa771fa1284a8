"""Per-op known-answer cases: a port of the reference's tests/wasm_plan.test.ts (every computation
of the WASM executor against a float64 computation on random inputs, with L and D outside
groups of 4, masked rows, NaN-poisoned padding rows and batches of two sequences).

Each case is a one-segment Plan in the IR of src/plan/ir.ts (the test's ``mini()`` helper,
tests/wasm_plan.test.ts:49-66), the buffer contents to write before the run, the rows to run,
the buffer to read and the float64 expectation (the formulas of the test file). Random inputs
come from the test's LCG (seed 12345, tests/wasm_plan.test.ts:13-18), drawn in the test file's
order. The same cases run against the oracle (tests/test_oracle_kat.py) and against the CUDA
backend (tests/test_gpu_kernels.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


class Lcg:
    """tests/wasm_plan.test.ts:13-18."""

    def __init__(self, seed: int = 12345):
        self.seed = seed

    def rand(self) -> float:
        self.seed = (self.seed * 1103515245 + 12345) & 0xFFFFFFFF
        return self.seed / 4294967296 * 2 - 1

    def arr(self, n: int, s: float = 1.0) -> np.ndarray:
        return np.array([self.rand() * s for _ in range(n)], dtype=np.float32)


def gelu64(v):
    """tests/wasm_plan.test.ts:22-28 (A&S 7.1.26 in f64)."""
    v = np.asarray(v, dtype=np.float64)
    u = v * math.sqrt(0.5)
    t = 1 / (1 + 0.3275911 * np.abs(u))
    p = (((((1.061405429 * t - 1.453152027) * t) + 1.421413741) * t - 0.284496736) * t + 0.254829592) * t
    e = 1 - p * np.exp(-u * u)
    return 0.5 * v * (1 + np.where(v >= 0, e, -e))


ACT = [lambda v: v, lambda v: np.maximum(v, 0), gelu64, np.tanh, lambda v: v / (1 + np.exp(-v))]


@dataclass
class Case:
    name: str
    plan: dict
    weights: dict = field(default_factory=dict)      # name -> (array, panel)
    writes: dict = field(default_factory=dict)       # buffer id -> array (written as raw bytes)
    rows: int = 1
    read: str = ""
    read_count: int = 0                              # f32 elements to compare
    want: np.ndarray | None = None
    tol: float = 2e-5
    mask_rows: np.ndarray | None = None              # rows whose output is compared only when set
    zero_rows: list = field(default_factory=list)    # (start, end) element ranges that must be exactly 0
    row_width: int = 0
    kernels: tuple = ()                              # plan kernels the case exercises


def mini(ops: list[dict], buffers: dict, L: int, out: str, batch: int = 1) -> dict:
    """tests/wasm_plan.test.ts:49-66: buffers given as element counts (f32) or init arrays."""
    decls = []
    for bid, v in buffers.items():
        if isinstance(v, (int, np.integer)):
            decls.append({"id": bid, "bytes": 4 * int(v), "usage": "rw"})
        else:
            a = np.ascontiguousarray(v)
            decls.append({"id": bid, "bytes": a.nbytes, "usage": "rw", "init": a.tobytes()})
    n_out = buffers[out]
    return {"f16": False, "length": L, "batch": batch, "markers": 0, "embeddingSize": 1, "buffers": decls,
            "segments": [{"name": "s", "prefix": "", "ops": ops}],
            "inputs": {"embeddings": "mask", "mask": "mask"},
            "output": {"buffer": out, "bytes": 4 * int(n_out), "dtype": "f32", "rows": int(n_out), "cols": 1},
            "captureSlots": 0, "captureSlotBytes": 0}


def prefix_mask(L: int, lens) -> np.ndarray:
    m = np.zeros(L * len(lens), dtype=np.float32)
    for b, n in enumerate(lens):
        m[b * L: b * L + n] = 1
    return m


def attention_ref(qkv, mask, L, B, H, D, scale, window, rows, rel=None):
    """tests/wasm_plan.test.ts:299-333 in numpy f64."""
    hd = H * D
    q64 = qkv.astype(np.float64)
    out = np.zeros(rows * hd)
    for i in range(rows):
        b, il = divmod(i, L)
        if mask[i] <= 0.5:
            continue
        for h in range(H):
            keys, s = [], []
            for j in range(L):
                if mask[b * L + j] <= 0.5 or (window and abs(il - j) > window):
                    continue
                q = q64[i * 3 * hd + h * D: i * 3 * hd + h * D + D]
                k = q64[(b * L + j) * 3 * hd + (H + h) * D: (b * L + j) * 3 * hd + (H + h) * D + D]
                v = float(q @ k)
                if rel is not None:
                    p = int(rel["idx"][il * L + j])
                    v += float(q @ rel["pk"][p * hd + h * D: p * hd + h * D + D].astype(np.float64))
                    v += float(k @ rel["pq"][p * hd + h * D: p * hd + h * D + D].astype(np.float64))
                keys.append(j)
                s.append(v / scale if rel is not None else v * scale)
            s = np.array(s)
            e = np.exp(s - s.max())
            pr = e / e.sum()
            for d in range(D):
                acc = 0.0
                for n, j in enumerate(keys):
                    acc += pr[n] * q64[(b * L + j) * 3 * hd + (2 * H + h) * D + d]
                out[i * hd + h * D + d] = acc
    return out


SPAN = 4


def rel_table(L: int) -> np.ndarray:
    """tests/wasm_plan.test.ts:336-340."""
    t = np.zeros(L * L, dtype=np.uint32)
    for i in range(L):
        for j in range(L):
            t[i * L + j] = min(max(i - j + SPAN, 0), 2 * SPAN - 1)
    return t


def all_cases(with_masklogits: bool = True) -> list[Case]:
    g = Lcg(12345)
    cases: list[Case] = []

    # matmul, tests/wasm_plan.test.ts:73-101
    for N, panel in ((37, True), (3, False), (16, True), (40, True)):
        M = 9 if N == 40 else 7
        K = 19
        W = g.arr(N * K)
        Bv = g.arr(N)
        for act in range(5):
            for fixed in (False, True):
                A = g.arr(M * K, 2)
                rows = M if fixed else 5
                want = ACT[act](A[:rows * K].reshape(rows, K).astype(np.float64) @
                                W.reshape(N, K).astype(np.float64).T + Bv.astype(np.float64))
                plan = mini([{"name": "mm", "kernel": "mmtile", "constants": {"M": M, "N": N, "K": K, "ACT": act},
                              "bind": ["a", "w:w", "w:b", "c"], "dispatch": [1, 1 if fixed else "rows32"]}],
                            {"mask": M, "a": M * K, "c": M * N}, M, "c")
                cases.append(Case(f"matmul N={N} act={act} fixed={fixed}", plan,
                                  {"w": (W.reshape(N, K), panel), "b": (Bv, False)}, {"a": A},
                                  1 if fixed else rows, "c", rows * N, want.reshape(-1), kernels=("mmtile",)))

    # layernorm modes and embln, tests/wasm_plan.test.ts:103-157
    N, rows = 21, 5
    w = g.arr(N)
    bias = g.arr(N)

    def ln_ref(v, scale):
        v = np.asarray(v, dtype=np.float64)
        mean = v.mean()
        var = ((v - mean) ** 2).mean()
        inv = 1 / math.sqrt(var + 1e-5)
        return ((v - mean) * inv * w + bias) * scale

    for mode in (0, 1, 2):
        a = g.arr(rows * N, 3)
        b = g.arr(rows * N, 3)
        mask = np.array([1, 1, 0, 1, 0], dtype=np.float32)
        want = []
        for r in range(rows):
            v = a[r * N:(r + 1) * N].astype(np.float64) + (b[r * N:(r + 1) * N] if mode == 2 else 0)
            want.append(ln_ref(v, mask[r] if mode == 1 else 1))
        plan = mini([{"name": "ln", "kernel": "layernorm", "constants": {"N": N, "MODE": mode, "EPS": 1e-5},
                      "bind": ["a", "b", "w:w", "w:bias", "mask", "o"], "dispatch": ["rows", 1]}],
                    {"mask": rows, "a": rows * N, "b": rows * N, "o": rows * N}, rows, "o")
        cases.append(Case(f"layernorm mode {mode}", plan, {"w": (w, False), "bias": (bias, False)},
                          {"a": a, "b": b, "mask": mask}, rows, "o", rows * N, np.concatenate(want),
                          kernels=("layernorm",)))
    L, P = 6, 9
    pos = g.arr(P * N)
    typ = g.arr(3 * N)
    for posids in (0, 1):
        for maskmul in (0, 1):
            word = g.arr(2 * L * N)
            types = np.array([(i % 3) | ((((i * 5) % P) << 16) if posids else 0) for i in range(2 * L)],
                             dtype=np.uint32)
            mask = prefix_mask(L, [4, 6])
            want = []
            for r in range(2 * L):
                prow = min(int(types[r] >> 16) if posids else (r % L) + 2, P - 1)
                v = (word[r * N:(r + 1) * N].astype(np.float64) + pos[prow * N:(prow + 1) * N]
                     + typ[int(types[r] & 0xFFFF) * N:(int(types[r] & 0xFFFF) + 1) * N])
                want.append(ln_ref(v, mask[r] if maskmul else 1))
            plan = mini([{"name": "e", "kernel": "embln",
                          "constants": {"N": N, "L": L, "OFFSET": 2, "MAXPOS": P, "EPS": 1e-5, "MASKMUL": maskmul,
                                        "POSIDS": posids},
                          "bind": ["word", "w:pos", "w:typ", "tt", "w:w", "w:bias", "mask", "o"],
                          "dispatch": ["rows", 1]}],
                        {"mask": 2 * L, "word": 2 * L * N, "tt": 2 * L, "o": 2 * L * N}, L, "o", batch=2)
            cases.append(Case(f"embln posids={posids} maskmul={maskmul}", plan,
                              {"pos": (pos.reshape(P, N), False), "typ": (typ.reshape(3, N), False),
                               "w": (w, False), "bias": (bias, False)},
                              {"word": word, "mask": mask, "tt": types}, 2 * L, "o", 2 * L * N, np.concatenate(want),
                              kernels=("embln",)))

    # add, gather, pool, geglu, rope, im2col, masklogits, tests/wasm_plan.test.ts:159-295
    L, N, B = 7, 6, 2
    for mode in (0, 1):
        d = g.arr(B * L * N)
        s = g.arr(B * L * N)
        idx = np.arange(B * L * N)
        want = d.astype(np.float64) + (s[(idx // (N * L)) * N + idx % N] if mode else s)
        plan = mini([{"name": "a", "kernel": "add", "constants": {"TOTAL": B * L * N, "N": N, "MODE": mode, "L": L},
                      "bind": ["dst", "src"], "dispatch": [1, 1]}],
                    {"mask": B * L, "dst": B * L * N, "src": B * L * N}, L, "dst", batch=B)
        cases.append(Case(f"add mode {mode}", plan, {}, {"dst": d, "src": s}, B * L, "dst", B * L * N, want,
                          kernels=("add",)))
    K = 3
    marks = np.array([2, 0, 5, 0, 0, 0, 0, 0, 0, 6, 1, 3, 0, 0, 0, 0, 0, 0], dtype=np.uint32)
    x = g.arr(B * L * N)
    want = []
    for gi in range(B * K):
        b = gi // K
        row = b * L + int(marks[b * 3 * K + gi - b * K])
        want.append(x[row * N:(row + 1) * N])
    plan = mini([{"name": "g", "kernel": "gather", "constants": {"K": K, "D": N, "L": L}, "bind": ["mk", "x", "st"],
                  "dispatch": [1, 1]}], {"mask": B * L, "mk": marks, "x": B * L * N, "st": B * K * N}, L, "st",
                batch=B)
    cases.append(Case("gather", plan, {}, {"x": x}, B * L, "st", B * K * N, np.concatenate(want).astype(np.float64),
                      kernels=("gather",)))
    for mode in (0, 1):
        x = g.arr(B * L * N)
        mask = prefix_mask(L, [3, 7])
        for r in range(B * L):
            if not mask[r]:
                x[r * N:(r + 1) * N] = np.nan
        want = []
        for b in range(B):
            vals = np.array([x[(b * L + i) * N:(b * L + i + 1) * N] for i in range(L) if mask[b * L + i]],
                            dtype=np.float64)
            want.append(vals.max(axis=0) if mode else vals.mean(axis=0))
        plan = mini([{"name": "p", "kernel": "pool", "constants": {"L": L, "N": N, "MODE": mode},
                      "bind": ["x", "mask", "o"], "dispatch": [1, B]}], {"mask": B * L, "x": B * L * N, "o": B * N},
                    L, "o", batch=B)
        cases.append(Case(f"pool mode {mode}", plan, {}, {"x": x, "mask": mask}, B * L, "o", B * N,
                          np.concatenate(want), kernels=("pool",)))
    I = 5
    mid = g.arr(L * 2 * I, 3)
    m2 = mid.reshape(L, 2 * I).astype(np.float64)
    want = (gelu64(m2[:, :I]) * m2[:, I:]).reshape(-1)
    plan = mini([{"name": "gg", "kernel": "geglu", "constants": {"I": I}, "bind": ["mid", "g"], "dispatch": ["rows", 1]}],
                {"mask": L, "mid": L * 2 * I, "g": L * I}, L, "g")
    cases.append(Case("geglu", plan, {}, {"mid": mid}, L, "g", L * I, want, kernels=("geglu",)))
    H, D = 2, 6
    table = np.zeros(L * 2 * D, dtype=np.float32)
    for i in range(L):
        for d in range(D // 2):
            f = i * 10000 ** (-(2 * d) / D)
            table[i * 2 * D + d] = math.cos(f)
            table[i * 2 * D + D + d] = math.sin(f)
    qkv = g.arr(B * L * 3 * H * D)
    want = qkv.astype(np.float64).copy()
    for i in range(B * L):
        il = i % L
        for s in range(2 * H):
            base = i * 3 * H * D + s * D
            for d in range(D // 2):
                xv, yv = float(qkv[base + d]), float(qkv[base + d + D // 2])
                c, sn = float(table[il * 2 * D + d]), float(table[il * 2 * D + D + d])
                want[base + d] = xv * c - yv * sn
                want[base + d + D // 2] = yv * c + xv * sn
    plan = mini([{"name": "r", "kernel": "rope", "constants": {"L": L, "H": H, "D": D}, "bind": ["qkv", "cs"],
                  "dispatch": ["rows", 2 * H]}], {"mask": B * L, "qkv": B * L * 3 * H * D, "cs": table}, L, "qkv",
                batch=B)
    cases.append(Case("rope", plan, {}, {"qkv": qkv}, B * L, "qkv", B * L * 3 * H * D, want, kernels=("rope",)))
    KS = 3
    x = g.arr(B * L * N)
    mask = prefix_mask(L, [5, 7])
    for r in range(B * L):
        if not mask[r]:
            x[r * N:(r + 1) * N] = np.nan
    want = []
    for r in range(B * L):
        for t in range(KS):
            j = (r % L) + t - 1
            src = (r // L) * L + max(j, 0)
            ok = 0 <= j < L and mask[src] != 0
            want.append(x[src * N:(src + 1) * N].astype(np.float64) if ok else np.zeros(N))
    plan = mini([{"name": "i", "kernel": "im2col", "constants": {"N": N, "L": L, "KS": KS}, "bind": ["x", "mask", "o"],
                  "dispatch": ["rows", 1]}], {"mask": B * L, "x": B * L * N, "o": B * L * KS * N}, L, "o", batch=B)
    cases.append(Case("im2col", plan, {}, {"x": x, "mask": mask}, B * L, "o", B * L * KS * N, np.concatenate(want),
                      kernels=("im2col",)))
    K = 4
    packed = np.zeros(3 * K * B, dtype=np.uint32)
    mbits = packed.view(np.float32)
    for k, v in enumerate([1, 0, 1, 1]):
        mbits[K + k] = v
    for k, v in enumerate([0, 1, 1, 0]):
        mbits[3 * K + K + k] = v
    raw = g.arr(B * K)
    want = np.array([raw[k] / 0.5 if mbits[(k // K) * 3 * K + K + k % K] > 0.5 else -1e4 for k in range(B * K)],
                    dtype=np.float64)
    if with_masklogits:
        plan = mini([{"name": "m", "kernel": "masklogits", "constants": {"K": K, "TEMP": 0.5},
                      "bind": ["raw", "pk", "lg"], "dispatch": [1, 1]}],
                    {"mask": B * L, "raw": B * K, "pk": packed, "lg": B * K}, L, "lg", batch=B)
        cases.append(Case("masklogits", plan, {}, {"raw": raw}, B * L, "lg", B * K, want, kernels=("masklogits",)))

    # attention, tests/wasm_plan.test.ts:342-401
    for L, D, lens, window in ((7, 5, [5], 0), (9, 6, [4, 9], 0), (9, 6, [9, 6], 2), (12, 8, [12], 0)):
        B = len(lens)
        H = 2
        hd = H * D
        rows = lens[0] if B == 1 else B * L
        qkv = g.arr(B * L * 3 * hd, 2)
        mask = prefix_mask(L, lens)
        for r in range(B * L):
            if not mask[r]:
                qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
        want = attention_ref(qkv, mask, L, B, H, D, 0.3, window, rows)
        base = {"L": L, "H": H, "D": D}
        for fused in ("split", "mbflash", "mbattention"):
            if fused == "split":
                ops = [{"name": "s", "kernel": "attscore", "constants": {**base, "SCALE": 0.3, "ROWS": B * L},
                        "bind": ["qkv", "ki", "sc"], "dispatch": [1, "rows32"]},
                       {"name": "p", "kernel": "attsoftmax", "constants": {"L": L, "H": H, "WINDOW": window},
                        "bind": ["mask", "sc"], "dispatch": [H, "rows"]},
                       {"name": "v", "kernel": "attpv", "constants": {**base, "ROWS": B * L},
                        "bind": ["sc", "qkv", "mask", "ki", "ctx"], "dispatch": [1, "rows32"]}]
            else:
                ops = [{"name": "a", "kernel": fused, "constants": {**base, "SCALE": 0.3, "WINDOW": window, "ROWS": B * L},
                        "bind": ["qkv", "mask", "ctx"], "dispatch": [H, "rows"]}]
            plan = mini(ops, {"mask": B * L, "qkv": B * L * 3 * hd, "ki": 2 * B, "sc": B * L * H * L,
                              "ctx": B * L * hd}, L, "ctx", batch=B)
            cases.append(Case(f"standard attention {fused} L={L} D={D} lens={lens} window={window}", plan, {},
                              {"qkv": qkv, "mask": mask}, rows, "ctx", rows * hd, want, mask_rows=mask[:rows],
                              row_width=hd, kernels=tuple(o["kernel"] for o in ops)))
        if window:
            continue
        qkv = g.arr(B * L * 3 * hd, 2)
        mask = prefix_mask(L, lens)
        for r in range(B * L):
            if not mask[r]:
                qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
        idx = rel_table(L)
        pk = g.arr(2 * SPAN * hd)
        pq = g.arr(2 * SPAN * hd)
        scale = math.sqrt(3 * D)
        want = attention_ref(qkv, mask, L, B, H, D, scale, 0, rows, {"idx": idx, "pk": pk, "pq": pq})
        moff = int(idx[L - 1])
        nm = int(idx[(L - 1) * L]) - moff + 1
        rel_c = {"H": H, "D": D, "ROWS": B * L, "NM": nm, "MOFF": moff, "L": L}
        for fused in (False, True):
            if fused:
                ops = [{"name": "a", "kernel": "attention", "constants": {"L": L, "H": H, "D": D, "SCALE": scale},
                        "bind": ["qkv", "w:pk", "w:pq", "ri", "mask", "ctx"], "dispatch": [H, "rows"]}]
            else:
                ops = [{"name": "c", "kernel": "attrel", "constants": {**rel_c, "PART": 0},
                        "bind": ["qkv", "w:pk", "ki", "ri", "c2p"], "dispatch": [1, "rows32"]},
                       {"name": "p", "kernel": "attrel", "constants": {**rel_c, "PART": 1},
                        "bind": ["qkv", "w:pq", "ki", "ri", "p2c"], "dispatch": [1, "rows32"]},
                       {"name": "s", "kernel": "attscore", "constants": {"L": L, "H": H, "D": D, "SCALE": 1 / scale,
                                                                          "ROWS": B * L},
                        "bind": ["qkv", "ki", "sc"], "dispatch": [1, "rows32"]},
                       {"name": "sr", "kernel": "attsoftrel",
                        "constants": {"L": L, "H": H, "NM": nm, "MOFF": moff, "INVSCALE": 1 / scale},
                        "bind": ["mask", "ri", "c2p", "p2c", "sc"], "dispatch": [H, "rows"]},
                       {"name": "v", "kernel": "attpv", "constants": {"L": L, "H": H, "D": D, "ROWS": B * L},
                        "bind": ["sc", "qkv", "mask", "ki", "ctx"], "dispatch": [1, "rows32"]}]
            plan = mini(ops, {"mask": B * L, "qkv": B * L * 3 * hd, "ki": 2 * B, "ri": idx, "sc": B * L * H * L,
                              "c2p": B * L * H * nm, "p2c": B * L * H * nm, "ctx": B * L * hd}, L, "ctx", batch=B)
            cases.append(Case(f"relative attention {'fused' if fused else 'split'} L={L} D={D} lens={lens}", plan,
                              {"pk": (pk.reshape(2 * SPAN, hd), False), "pq": (pq.reshape(2 * SPAN, hd), False)},
                              {"qkv": qkv, "mask": mask}, rows, "ctx", rows * hd, want, mask_rows=mask[:rows],
                              row_width=hd, kernels=tuple(o["kernel"] for o in ops)))
    return cases


def close(got: np.ndarray, want: np.ndarray, what: str, tol: float = 2e-5) -> None:
    """tests/wasm_plan.test.ts:30-38: |got - want| <= tol * max(1, max |want|), got finite."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{what}: length {got.shape} vs {want.shape}"
    scale = max(1.0, float(np.abs(want).max())) if want.size else 1.0
    bad = ~(np.isfinite(got) & (np.abs(got - want) <= tol * scale))
    if bad.any():
        i = int(np.argmax(bad))
        raise AssertionError(f"{what}[{i}]: {got[i]} vs {want[i]} ({int(bad.sum())} of {got.size} outside {tol})")


def check_case(case: Case, got: np.ndarray, tol: float | None = None) -> None:
    """Compares a run's output with the expectation as the reference test does: attention rows of
    masked queries are compared as zeros and must be exactly 0."""
    got = np.asarray(got, dtype=np.float64)[: case.read_count]
    t = case.tol if tol is None else tol
    if case.mask_rows is not None:
        w = case.row_width
        keep = np.repeat(case.mask_rows > 0, w)
        close(np.where(keep, got, 0.0), case.want, case.name, t)
        for r in np.nonzero(case.mask_rows == 0)[0]:
            seg = got[r * w:(r + 1) * w]
            assert np.all(seg == 0), f"{case.name}: masked row {r} not zero"
    else:
        close(got, case.want, case.name, t)

"""ORACLE — test infrastructure only (tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg). Nothing in the product imports this module.

Restatement of the host side of kleinhirn's WASM executor, ``src/plan/wasm.ts``:

- ``panel_weights``  = ``panelWeights``  (src/plan/wasm.ts:32-51)
- ``fuse_attention`` = ``fuseAttention`` (src/plan/wasm.ts:58-82)
- ``Runtime``        = ``WasmPlanRuntime`` (src/plan/wasm.ts:151-273): one byte arena for the
  weights and the plans, 64-byte aligned allocations with 64 spare bytes each, matmul
  weights with N >= 16 packed in panels [ceil(N / 16)][K][16].
- ``OraclePlan``     = ``WasmPlan`` (src/plan/wasm.ts:275-483): buffers at fixed addresses,
  per-thread scratch for the fused attention, the op stream (header of 8 words, 32-word
  records), upload, run, readOutput.

The stream is executed by ``oracle/wasm_plan.cpp`` (the restatement of src/wasm/plan.ts),
built into ``oracle/_build/liboracle.so`` by ``oracle/Makefile``.
"""
from __future__ import annotations

import ctypes
import math
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

HEAD = 8
OPW = 32
PAD = 64
NR = 16
CODE = {
    "gemmP": 1, "gemmNT": 2, "layernorm": 3, "embln": 4, "add": 5, "gather": 6, "pool": 7, "geglu": 8,
    "rope": 9, "im2col": 10, "attscore": 11, "attsoftmax": 12, "attpv": 13, "attrel": 14, "attsoftrel": 15,
    "attstd": 16, "attrelf": 17, "masklogits": 18,
}
MATMUL = {"matmul", "mmtile", "mmtile8", "mmtile16"}
DEFAULT_SPLIT = {"rb": 16, "cb": 64, "qb": 32, "minWork": 1 << 16}  # src/plan/wasm.ts:124

_lib = None


def build() -> Path:
    """Compiles the oracle with its Makefile (gcc -O3 -march=native -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.oracle_run.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p]
        _lib.oracle_run_range.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_void_p]
        _lib.oracle_threads_create.argtypes = [ctypes.c_int] * 5
        _lib.oracle_threads_create.restype = ctypes.c_void_p
        _lib.oracle_threads_destroy.argtypes = [ctypes.c_void_p]
        for f in ("oracle_vexp1", "oracle_vgelu1", "oracle_gelu"):
            getattr(_lib, f).argtypes = [ctypes.c_float]
            getattr(_lib, f).restype = ctypes.c_float
    return _lib


def _align(n: int) -> int:
    return math.ceil(n / 64) * 64


def panel_weights(plans: list[dict]) -> set[str]:
    """src/plan/wasm.ts:32-51."""
    role: dict[str, str] = {}
    for plan in plans:
        for seg in plan["segments"]:
            for op in seg["ops"]:
                for i, bid in enumerate(op["bind"]):
                    if not bid.startswith("w:"):
                        continue
                    name = bid[2:]
                    r = ("kn" if op["constants"]["N"] >= 16 else "nk") if (op["kernel"] in MATMUL and i == 1) else "plain"
                    was = role.get(name)
                    if was is not None and was != r:
                        raise ValueError(f"weight {name} is bound as {was} and as {r}")
                    role[name] = r
    return {n for n, r in role.items() if r == "kn"}


def fuse_attention(ops: list[dict]) -> list[dict]:
    """src/plan/wasm.ts:58-82."""
    out = []
    k = lambda i: ops[i]["kernel"] if i < len(ops) else None  # noqa: E731
    i = 0
    while i < len(ops):
        o = ops[i]
        if (o["kernel"] == "attscore" and k(i + 1) == "attsoftmax" and k(i + 2) == "attpv"
                and ops[i + 1]["bind"][1] == o["bind"][2] and ops[i + 2]["bind"][0] == o["bind"][2]):
            c = o["constants"]
            out.append({"name": f"{o['name']}+fused", "kernel": "mbattention",
                        "constants": {"L": c["L"], "H": c["H"], "D": c["D"], "SCALE": c["SCALE"],
                                      "WINDOW": ops[i + 1]["constants"]["WINDOW"]},
                        "bind": [o["bind"][0], ops[i + 1]["bind"][0], ops[i + 2]["bind"][4]],
                        "dispatch": o["dispatch"]})
            i += 3
        elif (o["kernel"] == "attrel" and o["constants"]["PART"] == 0 and k(i + 1) == "attrel"
              and ops[i + 1]["constants"]["PART"] == 1 and k(i + 2) == "attscore" and k(i + 3) == "attsoftrel"
              and k(i + 4) == "attpv"):
            s = ops[i + 2]
            out.append({"name": f"{s['name']}+fused", "kernel": "attention",
                        "constants": {"L": s["constants"]["L"], "H": s["constants"]["H"], "D": s["constants"]["D"],
                                      "SCALE": 1 / s["constants"]["SCALE"]},
                        "bind": [o["bind"][0], o["bind"][1], ops[i + 1]["bind"][1], o["bind"][3],
                                 ops[i + 3]["bind"][0], ops[i + 4]["bind"][4]],
                        "dispatch": s["dispatch"]})
            i += 5
        else:
            out.append(o)
            i += 1
    return out


class Runtime:
    """src/plan/wasm.ts:151-273 (single arena, optional helper threads)."""

    def __init__(self, threads: int = 1, split: dict | None = None):
        self.mem = np.zeros(1 << 20, dtype=np.uint8)
        self.top = 64
        self.addr: dict[str, int] = {}
        self.panels: set[str] = set()
        self.weight_bytes = 0
        self.threads = max(1, threads)
        s = split or DEFAULT_SPLIT
        self.pool = lib().oracle_threads_create(self.threads, s["rb"], s["cb"], s["qb"], s["minWork"]) \
            if self.threads > 1 else None

    def close(self):
        if self.pool:
            lib().oracle_threads_destroy(self.pool)
            self.pool = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def alloc(self, nbytes: int) -> int:
        p = self.top
        self.top = _align(p + nbytes + PAD)
        if self.top > self.mem.size:
            if self.top >= 1 << 32:
                raise MemoryError("oracle arena exceeds 4 GiB (u32 addresses)")
            new = np.zeros(max(self.top, 2 * self.mem.size), dtype=np.uint8)
            new[: self.mem.size] = self.mem
            self.mem = new
        return p

    def f32(self, p: int, n: int) -> np.ndarray:
        return self.mem[p: p + 4 * n].view(np.float32)

    def add_weight(self, name: str, shape, data: np.ndarray, panel: bool) -> None:
        """src/plan/wasm.ts:232-255."""
        if name in self.addr:
            raise ValueError(f"weight {name} loaded twice")
        data = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        nbytes = data.nbytes
        if panel:
            if len(shape) != 2 or shape[0] * shape[1] != data.size:
                raise ValueError(f"weight {name}: shape {shape} is no matrix")
            N, K = shape
            nbytes = 4 * math.ceil(N / NR) * NR * K
        p = self.alloc(nbytes)
        dst = self.f32(p, nbytes // 4)
        if panel:
            N, K = shape
            dst[:] = 0
            w = data.reshape(N, K)
            np_ = math.ceil(N / NR)
            pad = np.zeros((np_ * NR, K), dtype=np.float32)
            pad[:N] = w
            # [ceil(N/16)][K][16]: element (n, k) at (n // 16) * K * 16 + k * 16 + n % 16
            dst[:] = pad.reshape(np_, NR, K).transpose(0, 2, 1).reshape(-1)
        else:
            dst[:] = data
        self.addr[f"w:{name}"] = p
        if panel:
            self.panels.add(f"w:{name}")
        self.weight_bytes += _align(nbytes + PAD)

    def weight(self, bid: str):
        return self.addr.get(bid)

    def paneled(self, bid: str) -> bool:
        return bid in self.panels

    def plan(self, plan: dict) -> "OraclePlan":
        if plan["f16"]:
            raise ValueError("the WASM executor runs f32 plans")
        return OraclePlan(self, plan)


class OraclePlan:
    """src/plan/wasm.ts:275-483."""

    def __init__(self, rt: Runtime, plan: dict):
        self.rt = rt
        self.plan = plan
        self.length = plan["length"]
        self.batch = plan["batch"]
        ops = fuse_attention([op for s in plan["segments"] for op in s["ops"]])
        used = {b for o in ops for b in o["bind"]} | {plan["output"]["buffer"]} | \
            {v for v in plan["inputs"].values() if isinstance(v, str)}
        if plan.get("rowSelect"):  # src/plan/wasm.ts:291
            used.add(plan["rowSelect"]["dst"])
        self.bufs: dict[str, tuple[int, int]] = {}
        for d in plan["buffers"]:
            if d["id"] not in used:
                continue
            p = rt.alloc(d["bytes"])
            self.bufs[d["id"]] = (p, d["bytes"])
            if d.get("init") is not None:
                init = np.frombuffer(bytes(d["init"]), dtype=np.uint8)
                rt.mem[p: p + init.size] = init
        self.ops = ops
        L = plan["length"]
        scratch = max([0] + [(5 * L * L + (2 * L + 16) * o["constants"]["D"]) if o["kernel"] == "attention"
                             else (L * L + (L + 16) * o["constants"]["D"]) if o["kernel"] in ("mbattention", "mbflash")
                             else 0 for o in ops])
        kinfo = rt.alloc(8 * plan["batch"])
        scratch_bytes = _align(4 * scratch)
        scratch_p = rt.alloc(scratch_bytes * rt.threads) if scratch else 0
        self.stream = rt.alloc(4 * (HEAD + OPW * len(ops)))
        words = np.zeros(HEAD + OPW * len(ops), dtype=np.int32)
        words[:HEAD] = [len(ops), L, plan["batch"], self._at(plan["inputs"]["mask"]), kinfo, scratch_p,
                        scratch_bytes, 0]
        for i, op in enumerate(ops):
            self._encode(op, words, HEAD + OPW * i)
        rt.mem[self.stream: self.stream + words.nbytes] = words.view(np.uint8)

    def _at(self, bid: str) -> int:
        p = self.rt.weight(bid) if bid.startswith("w:") else self.bufs.get(bid, (None,))[0]
        if p is None:
            raise ValueError(f"wasm plan: {'weight' if bid.startswith('w:') else 'buffer'} {bid} missing")
        return p

    def _bytes(self, bid: str) -> int:
        return self.bufs[bid][1]

    def _encode(self, op: dict, w: np.ndarray, o: int) -> None:
        """src/plan/wasm.ts:330-407."""
        c = op["constants"]
        for i, bid in enumerate(op["bind"]):
            if self.rt.paneled(bid) and not (op["kernel"] in MATMUL and i == 1):
                raise ValueError(f"wasm plan: {op['name']} reads the paneled weight {bid} as a plain tensor")
        b = lambda i: self._at(op["bind"][i])  # noqa: E731
        fixed = lambda d, n: n if isinstance(d, int) else -1  # noqa: E731
        F = lambda v: ("f", v)  # noqa: E731
        k = op["kernel"]
        if k in MATMUL:
            rec = [CODE["gemmP"] if self.rt.paneled(op["bind"][1]) else CODE["gemmNT"], fixed(op["dispatch"][1], c["M"]),
                   b(0), b(1), b(2), b(3), c["N"], c["K"], c["ACT"], c["M"]]
        elif k == "layernorm":
            d0 = op["dispatch"][0]
            rec = [CODE["layernorm"], fixed(d0, d0), b(0), b(1), b(2), b(3), b(4), b(5), c["N"], c["MODE"], F(c["EPS"])]
        elif k == "embln":
            rec = [CODE["embln"], -1, b(0), b(1), b(2), b(3), b(4), b(5), b(6), b(7), c["N"], c["L"], c["OFFSET"],
                   c["MAXPOS"], F(c["EPS"]), c["MASKMUL"], c["POSIDS"]]
        elif k == "add":
            rec = [CODE["add"], -1, b(0), b(1), c["TOTAL"], c["N"], c["MODE"], c["L"]]
        elif k == "gather":
            rec = [CODE["gather"], -1, b(0), b(1), b(2), c["K"], c["D"], c["L"], self._bytes(op["bind"][0]) // 12]
        elif k == "pool":
            rec = [CODE["pool"], -1, b(0), b(1), b(2), c["L"], c["N"], c["MODE"], op["dispatch"][1]]
        elif k == "geglu":
            rec = [CODE["geglu"], -1, b(0), b(1), c["I"]]
        elif k == "rope":
            rec = [CODE["rope"], -1, b(0), b(1), c["L"], c["H"], c["D"]]
        elif k == "im2col":
            rec = [CODE["im2col"], -1, b(0), b(1), b(2), c["N"], c["L"], c["KS"]]
        elif k == "attscore":
            rec = [CODE["attscore"], -1, b(0), b(2), c["L"], c["H"], c["D"], F(c["SCALE"])]
        elif k == "attsoftmax":
            rec = [CODE["attsoftmax"], -1, b(0), b(1), c["L"], c["H"], c["WINDOW"]]
        elif k == "attpv":
            rec = [CODE["attpv"], -1, b(0), b(1), b(4), c["L"], c["H"], c["D"]]
        elif k == "attrel":
            rec = [CODE["attrel"], -1, b(0), b(1), b(3), b(4), c["H"], c["D"], c["NM"], c["MOFF"], c["PART"], c["L"]]
        elif k == "attsoftrel":
            rec = [CODE["attsoftrel"], -1, b(0), b(1), b(2), b(3), b(4), c["L"], c["H"], c["NM"], c["MOFF"],
                   F(c["INVSCALE"])]
        elif k in ("mbattention", "mbflash"):
            rec = [CODE["attstd"], -1, b(0), b(1), b(2), c["L"], c["H"], c["D"], F(c["SCALE"]), c["WINDOW"]]
        elif k == "attention":
            rec = [CODE["attrelf"], -1, b(0), b(1), b(2), b(3), b(4), b(5), c["L"], c["H"], c["D"], F(c["SCALE"])]
        elif k == "masklogits":
            rec = [CODE["masklogits"], -1, b(0), b(1), b(2), c["K"], F(c["TEMP"]), self._bytes(op["bind"][1]) // 12]
        else:
            raise ValueError(f"wasm plan: kernel {k} has no computation")
        for i, v in enumerate(rec):
            if isinstance(v, tuple):
                w[o + i] = np.array([v[1]], dtype=np.float32).view(np.int32)[0]
            else:
                if int(v) != v:
                    raise ValueError(f"wasm plan: {op['name']} argument {i} is {v}")
                w[o + i] = np.int64(v).astype(np.int32)

    def buf_view(self, bid: str) -> np.ndarray:
        p, n = self.bufs[bid]
        return self.rt.mem[p: p + n]

    def view(self, bid: str) -> np.ndarray:
        p, n = self.bufs[bid]
        return self.rt.f32(p, n // 4)

    def upload(self, embeddings: np.ndarray, mask: np.ndarray, type_ids: np.ndarray | None = None,
               packed_markers: np.ndarray | None = None, qtype=None) -> None:
        """src/plan/wasm.ts:409-440 (f32 word rows only): inputs, marker payload, Julia type rows."""
        i = self.plan["inputs"]

        def put(bid, src: np.ndarray):
            p, n = self.bufs[bid]
            raw = np.ascontiguousarray(src).view(np.uint8).reshape(-1)
            if raw.size > n:
                raise ValueError(f"wasm plan: input {bid} has {raw.size} B, the buffer {n}")
            self.rt.mem[p: p + raw.size] = raw
        if embeddings.dtype != np.float32:
            raise ValueError("the WASM executor takes f32 word rows")
        put(i["embeddings"], embeddings)
        put(i["mask"], mask.astype(np.float32))
        if i.get("markers"):
            if packed_markers is None:
                raise ValueError("plan needs packedMarkers")
            put(i["markers"], np.asarray(packed_markers, dtype=np.uint32))
        if i.get("typeIds"):
            if type_ids is None:
                raise ValueError("plan needs typeIds")
            put(i["typeIds"], type_ids.astype(np.uint32))
        rs = self.plan.get("rowSelect")
        if rs:
            qtypes = list(qtype) if isinstance(qtype, (list, tuple, np.ndarray)) else [qtype or 0]
            table, dst, rb = self._at(rs["table"]), self._at(rs["dst"]), rs["rowBytes"]
            for b in range(self.batch):
                q = int(qtypes[b]) if b < len(qtypes) else 0
                self.rt.mem[dst + b * rb: dst + (b + 1) * rb] = self.rt.mem[table + q * rb: table + (q + 1) * rb]

    def run(self, rows: int) -> None:
        if rows < 1 or rows > self.length * self.batch:
            raise ValueError(f"wasm plan: {rows} rows, the plan has {self.length * self.batch}")
        mem = self.rt.mem
        lib().oracle_run(mem.ctypes.data, self.stream, rows, self.rt.pool)

    def read_output(self) -> np.ndarray:
        o = self.plan["output"]
        p, _ = self.bufs[o["buffer"]]
        return self.rt.f32(p, o["rows"] * o["cols"]).copy()


def load_weights(rt: Runtime, tensors: dict[str, np.ndarray], plans: list[dict]) -> None:
    """Adds every non-word tensor in f32 (the word table stays on the host, src/wasm-backend.ts:184),
    packed in panels where a plan reads it as a matmul weight with N >= 16."""
    panels = panel_weights(plans)
    for name, arr in tensors.items():
        if name == "embeddings.word.weight":
            continue
        rt.add_weight(name, list(arr.shape), np.asarray(arr, dtype=np.float32), name in panels)

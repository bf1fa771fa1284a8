"""CudaBackend: kleinhirn's ``Backend`` / ``PlanRunner`` interface (src/backend.ts:14-46) over the
C ABI of libkhcuda.so (include/kh_cuda.h), through ctypes.

This is the Python twin of the N-API binding a Node host would use. Method names follow the
reference interface in snake_case:

    Backend.kind / weightBytes / check / runner / fitBatch / prepare / call / info / dispose
    PlanRunner.length / batch / markers / bytes / upload / run / readOutput / readCapture /
               assertCapturable / destroy

A non-zero status of the library raises ``KhError`` with the library's message, as the WASM
backend's ``answer()`` throws the worker's message (src/wasm-backend.ts:48-51). There is no
CPU fallback: if libkhcuda.so or a CUDA device is missing, construction fails.
"""
from __future__ import annotations

import ctypes
import json
import weakref
from pathlib import Path

import numpy as np

from .plan import plan_to_json

LIB_PATH = Path(__file__).resolve().parent / "libkhcuda.so"
KH_F32, KH_F16 = 0, 1
STATUS = {0: "ok", 1: "argument", 2: "plan", 3: "cuda", 4: "latched device error"}

# Every function of include/kh_cuda.h with its ctypes signature.
_P = ctypes.c_void_p
_SIGS = {
    "kh_last_error": ([], ctypes.c_char_p),
    "kh_init": ([ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.POINTER(_P)], ctypes.c_int),
    "kh_add_tensor": ([_P, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_int, _P,
                       ctypes.c_size_t], ctypes.c_int),
    "kh_add_words": ([_P, ctypes.c_char_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _P,
                      ctypes.c_size_t], ctypes.c_int),
    "kh_weight_bytes": ([_P], ctypes.c_int64),
    "kh_check": ([_P, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_int),
    "kh_plan_create": ([_P, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(_P)], ctypes.c_int),
    "kh_plan_info": ([_P, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                      ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "kh_upload": ([_P, _P, ctypes.c_size_t, _P, ctypes.c_size_t, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_upload_markers": ([_P, _P, ctypes.c_size_t, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_capture_check": ([_P], ctypes.c_int),
    "kh_run_capture": ([_P], ctypes.c_int),
    "kh_read_capture": ([_P, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_run": ([_P, ctypes.c_int], ctypes.c_int),
    "kh_read_output": ([_P, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_plan_destroy": ([_P], None),
    "kh_destroy": ([_P], None),
    "kh_info": ([_P, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_size_t),
    "kh_plan_launches": ([_P, ctypes.c_char_p, ctypes.c_size_t], ctypes.c_size_t),
    "kh_profile": ([_P, ctypes.c_int, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_plan_buffer_write": ([_P, ctypes.c_char_p, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_plan_buffer_read": ([_P, ctypes.c_char_p, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_bulk_create": ([_P, ctypes.c_int64, ctypes.c_int, ctypes.c_int64, ctypes.POINTER(_P)], ctypes.c_int),
    "kh_bulk_set_lengths": ([_P, _P, ctypes.c_int], ctypes.c_int),
    "kh_bulk_upload": ([_P, _P, ctypes.c_size_t, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_bulk_set_word_table": ([_P, ctypes.c_char_p], ctypes.c_int),
    "kh_bulk_upload_ids": ([_P, _P, ctypes.c_size_t, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_bulk_run": ([_P], ctypes.c_int),
    "kh_bulk_read": ([_P, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_run_batch": ([_P, _P, ctypes.c_int, _P, ctypes.c_size_t, _P, ctypes.c_size_t, _P, ctypes.c_size_t],
                     ctypes.c_int),
    "kh_bulk_last_timing": ([_P, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "kh_bulk_destroy": ([_P], None),
    "kh_bulk_profile": ([_P, _P, ctypes.c_size_t], ctypes.c_int),
    "kh_ctx_stream": ([_P], ctypes.c_void_p),
    "kh_attention_f16_noalloc": ([_P, _P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                  ctypes.c_int, _P], ctypes.c_int),
    "kh_attention_f16_noalloc_status": ([_P], ctypes.c_int),
    "kh_inject_cuda_error": ([_P, ctypes.c_char_p], ctypes.c_int),
    "kh_selftest_wait_limit": ([_P, ctypes.c_int], ctypes.c_int),
    "kh_selftest_tensor_maps": ([ctypes.c_int, ctypes.c_int], ctypes.c_int64),
}

_lib = None


class KhError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} [{STATUS.get(status, status)}]")
        self.status = status


def load_library(path: Path | str | None = None):
    """Loads libkhcuda.so (built in-tree by kleinhirn_b200.build) and declares every entry point."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: build it with python -m kleinhirn_b200.build")
    lib = ctypes.CDLL(str(p))
    for name, (args, res) in _SIGS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    if path is None:
        _lib = lib
    return lib


def _check(lib, status: int) -> None:
    if status != 0:
        raise KhError(status, lib.kh_last_error().decode("utf-8", "replace"))


def attention_f16_noalloc(qkv_ptr: int, mask_ptr: int, ctx_ptr: int, seq_lens, heads: int, head_dim: int,
                          scale: float, window: int = 0, stream: int = 0) -> None:
    """kh_attention_f16_noalloc on device pointers (qkv f16 [T, 3 H D], mask f32 [T], ctx f16 [T, H D]);
    seq_lens on the host, T = their sum. Queues the work on `stream` and allocates no device memory."""
    lib = load_library()
    lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    _check(lib, lib.kh_attention_f16_noalloc(qkv_ptr, mask_ptr, ctx_ptr, lens.ctypes.data, len(lens), heads,
                                              head_dim, scale, window, stream or None))


def attention_f16_noalloc_status(stream: int = 0) -> None:
    """kh_attention_f16_noalloc_status: waits for `stream`; raises KhError if an attention
    pipeline wait on the current device gave up since the last report (the report clears it)."""
    lib = load_library()
    _check(lib, lib.kh_attention_f16_noalloc_status(stream or None))


def selftest_tensor_maps(threads: int, iters: int) -> int:
    """kh_selftest_tensor_maps: descriptors that differ from a fresh encoding (0 expected)."""
    lib = load_library()
    n = int(lib.kh_selftest_tensor_maps(threads, iters))
    if n < 0:
        raise KhError(3, lib.kh_last_error().decode("utf-8", "replace"))
    return n


def _ptr(a: np.ndarray | None):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _string(fn, handle) -> str:
    n = fn(handle, None, 0)
    buf = ctypes.create_string_buffer(n)
    fn(handle, buf, n)
    return buf.value.decode()


class CudaPlanRunner:
    """PlanRunner (src/backend.ts:14-28) of one Plan on the device."""

    def __init__(self, backend: "CudaBackend", plan: dict):
        self.backend = backend
        self.lib = backend.lib
        self.plan = plan
        js = plan_to_json(plan).encode()
        h = ctypes.c_void_p()
        _check(self.lib, self.lib.kh_plan_create(backend.handle, js, len(js), ctypes.byref(h)))
        self.handle = h
        L, B, r, c, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        _check(self.lib, self.lib.kh_plan_info(h, ctypes.byref(L), ctypes.byref(B), ctypes.byref(r), ctypes.byref(c),
                                               ctypes.byref(nb)))
        self.length, self.batch = L.value, B.value
        self.out_rows, self.out_cols = r.value, c.value
        self.markers = plan["markers"]
        self._bytes = nb.value
        self.f16 = plan["f16"]
        self._bulks = weakref.WeakSet()  # open bulk handles: kh_plan_destroy frees them
        backend._runners.add(self)

    @property
    def bytes(self) -> int:
        return self._bytes

    def upload(self, embeddings: np.ndarray, mask: np.ndarray, type_ids: np.ndarray | None = None,
               packed_markers: np.ndarray | None = None, qtype=None) -> None:
        """RunInput (src/plan/executor.ts:25-37): embeddings f16 (or f16 bits as uint16) for f16 plans,
        f32 otherwise; mask f32; typeIds u32; for GLiNER2 / Julia plans packedMarkers u32 (3 K per
        sequence) and qtype (an int, or one per sequence)."""
        want = np.float16 if self.f16 else np.float32
        emb = np.ascontiguousarray(embeddings)
        if emb.dtype == np.uint16 and self.f16:
            emb = emb.view(np.float16)
        if emb.dtype != want:
            raise TypeError(f"embeddings must be {np.dtype(want).name} for this plan, got {emb.dtype}")
        m = np.ascontiguousarray(mask, dtype=np.float32)
        t = None if type_ids is None else np.ascontiguousarray(type_ids, dtype=np.uint32)
        _check(self.lib, self.lib.kh_upload(self.handle, _ptr(emb), emb.nbytes, _ptr(m), m.size, _ptr(t),
                                            0 if t is None else t.size))
        if packed_markers is not None or "markers" in self.plan["inputs"]:
            if packed_markers is None:
                raise KhError(1, "plan needs packedMarkers")
            pk = np.ascontiguousarray(packed_markers, dtype=np.uint32)
            q = None
            if qtype is not None:
                q = np.ascontiguousarray(np.atleast_1d(np.asarray(qtype)), dtype=np.int32)
            _check(self.lib, self.lib.kh_upload_markers(self.handle, _ptr(pk), pk.size, _ptr(q),
                                                        0 if q is None else q.size))

    def run(self, seq_len: int, capture: bool = False) -> None:
        """One forward over seq_len rows; with capture, over the full bucket, filling the capture
        slots (src/plan/executor.ts:232, :267-281)."""
        if capture:
            self.assert_capturable()
            _check(self.lib, self.lib.kh_run_capture(self.handle))
            return
        _check(self.lib, self.lib.kh_run(self.handle, int(seq_len)))

    def read_output(self) -> np.ndarray:
        out = np.empty(self.out_rows * self.out_cols, dtype=np.float32)
        _check(self.lib, self.lib.kh_read_output(self.handle, _ptr(out), out.size))
        return out

    def read_capture(self) -> np.ndarray:
        """captureSlots x captureSlotBytes / 4 f32 values of the last capture run
        (src/plan/executor.ts:418-424)."""
        self.assert_capturable()
        out = np.empty(self.plan.get("captureSlots", 0) * self.plan.get("captureSlotBytes", 0) // 4,
                       dtype=np.float32)
        _check(self.lib, self.lib.kh_read_capture(self.handle, _ptr(out), out.size))
        return out

    def assert_capturable(self) -> None:
        """Throws unless the plan can capture: f32 and batch 1 (src/plan/executor.ts:178-186)."""
        _check(self.lib, self.lib.kh_capture_check(self.handle))

    def write_buffer(self, bid: str, data: np.ndarray) -> None:
        """Raw bytes into a plan buffer (WasmPlan.view for tests, src/plan/wasm.ts:473-476)."""
        a = np.ascontiguousarray(data)
        _check(self.lib, self.lib.kh_plan_buffer_write(self.handle, bid.encode(), _ptr(a), a.nbytes))

    def read_buffer(self, bid: str, nbytes: int) -> np.ndarray:
        out = np.empty(nbytes, dtype=np.uint8)
        _check(self.lib, self.lib.kh_plan_buffer_read(self.handle, bid.encode(), _ptr(out), nbytes))
        return out

    def launches(self) -> list[dict]:
        return json.loads(_string(self.lib.kh_plan_launches, self.handle))

    def profile(self, rows: int) -> list[tuple[str, float]]:
        steps = self.launches()
        ms = np.zeros(len(steps), dtype=np.float32)
        _check(self.lib, self.lib.kh_profile(self.handle, int(rows), _ptr(ms), ms.size))
        return [(s["label"] + ":" + "+".join(s["ops"]), float(t)) for s, t in zip(steps, ms)]

    def destroy(self) -> None:
        if self.handle:
            self.lib.kh_plan_destroy(self.handle)
            self._forget()

    def _forget(self) -> None:
        """The library freed this plan (and its bulk handles): drop the handles."""
        self.handle = None
        for b in list(self._bulks):
            b.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class CudaBulk:
    """Ragged bulk runs of one plan (kh_bulk_*): sequences packed back to back, no padding rows."""

    def __init__(self, runner: CudaPlanRunner, max_tokens: int, max_seqs: int, chunk_tokens: int = 65536):
        self.runner = runner
        self.lib = runner.lib
        h = ctypes.c_void_p()
        _check(self.lib, self.lib.kh_bulk_create(runner.handle, int(max_tokens), int(max_seqs),
                                                 int(max(chunk_tokens, runner.length)), ctypes.byref(h)))
        self.handle = h
        self.n = 0
        self.tokens = 0
        runner._bulks.add(self)

    def set_lengths(self, lens) -> None:
        a = np.ascontiguousarray(lens, dtype=np.int32)
        _check(self.lib, self.lib.kh_bulk_set_lengths(self.handle, _ptr(a), a.size))
        self.n = a.size
        self.tokens = int(a.sum())

    def upload(self, emb: np.ndarray, type_ids: np.ndarray | None = None) -> None:
        e = np.ascontiguousarray(emb)
        t = None if type_ids is None else np.ascontiguousarray(type_ids, dtype=np.uint32)
        _check(self.lib, self.lib.kh_bulk_upload(self.handle, _ptr(e), e.nbytes, _ptr(t), 0 if t is None else t.size))

    def run(self) -> None:
        _check(self.lib, self.lib.kh_bulk_run(self.handle))

    def read(self) -> np.ndarray:
        rows = self.n if self.runner.out_rows <= self.runner.batch else self.tokens
        out = np.empty((rows, self.runner.out_cols), dtype=np.float32)
        _check(self.lib, self.lib.kh_bulk_read(self.handle, _ptr(out), out.size))
        return out

    def run_batch(self, lens, emb: np.ndarray, type_ids: np.ndarray | None = None) -> np.ndarray:
        self.set_lengths(lens)
        self.upload(emb, type_ids)
        self.run()
        return self.read()

    def profile(self) -> list[tuple[dict, float]]:
        """Per-step device ms of one bulk forward (summed over chunks), with the launch list."""
        steps = self.runner.launches()
        ms = np.zeros(len(steps), dtype=np.float32)
        _check(self.lib, self.lib.kh_bulk_profile(self.handle, _ptr(ms), ms.size))
        return list(zip(steps, ms.tolist()))

    def upload_ptr(self, emb_ptr: int, emb_bytes: int, type_ptr: int | None, type_len: int) -> None:
        """Upload from raw host pointers (pinned buffers of the caller)."""
        _check(self.lib, self.lib.kh_bulk_upload(self.handle, ctypes.c_void_p(emb_ptr), emb_bytes,
                                                 None if type_ptr is None else ctypes.c_void_p(type_ptr), type_len))

    def read_ptr(self, out_ptr: int, n: int) -> None:
        _check(self.lib, self.lib.kh_bulk_read(self.handle, ctypes.c_void_p(out_ptr), n))

    def set_word_table(self, name: str) -> None:
        """Keep the added tensor `name` ([vocab, embeddingSize]) as the device word table."""
        _check(self.lib, self.lib.kh_bulk_set_word_table(self.handle, name.encode()))

    def upload_ids(self, ids: np.ndarray, type_ids: np.ndarray | None = None) -> None:
        """Packed token ids of the sequences set last; word rows are gathered on the device."""
        i = np.ascontiguousarray(ids, dtype=np.int32)
        t = None if type_ids is None else np.ascontiguousarray(type_ids, dtype=np.uint32)
        _check(self.lib, self.lib.kh_bulk_upload_ids(self.handle, _ptr(i), i.size, _ptr(t), 0 if t is None else t.size))

    def upload_ids_ptr(self, ids_ptr: int, n: int, type_ptr: int | None, type_len: int) -> None:
        """upload_ids from raw host pointers (pinned buffers of the caller)."""
        _check(self.lib, self.lib.kh_bulk_upload_ids(self.handle, ctypes.c_void_p(ids_ptr), n,
                                                     None if type_ptr is None else ctypes.c_void_p(type_ptr),
                                                     type_len))

    def last_timing(self) -> tuple[float, int]:
        ms, n = ctypes.c_float(), ctypes.c_int64()
        _check(self.lib, self.lib.kh_bulk_last_timing(self.handle, ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    def close(self) -> None:
        if self.handle and self.runner.handle:
            self.lib.kh_bulk_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaBackend:
    """Backend (src/backend.ts:30-46) on one B200. ``tensors`` maps the manifest's tensor names to
    arrays (f32 or f16); the word table stays on the host (src/wasm-backend.ts:184)."""

    kind = "cuda"

    def __init__(self, tensors: dict[str, np.ndarray] | None = None, device: int = 0, lib_path=None):
        self.lib = load_library(lib_path)
        self._runners = weakref.WeakSet()  # open plans: kh_destroy frees them
        devs = (ctypes.c_int * 1)(device)
        h = ctypes.c_void_p()
        _check(self.lib, self.lib.kh_init(devs, 1, ctypes.byref(h)))
        self.handle = h
        for name, arr in (tensors or {}).items():
            if name == "embeddings.word.weight":
                continue
            self.add_tensor(name, arr)

    def add_words(self, name: str, words_bin: bytes | np.ndarray, dtype: str, rows: int, width: int,
                  row_bytes: int) -> None:
        """The word table from words.bin bytes (rows of `row_bytes`: values, then a checksum word)."""
        b = np.frombuffer(words_bin, dtype=np.uint8) if isinstance(words_bin, (bytes, bytearray)) else \
            np.ascontiguousarray(words_bin).view(np.uint8).reshape(-1)
        _check(self.lib, self.lib.kh_add_words(self.handle, name.encode(), KH_F16 if dtype == "f16" else KH_F32,
                                               rows, width, row_bytes, _ptr(b), b.size))

    def add_tensor(self, name: str, arr: np.ndarray) -> None:
        a = np.ascontiguousarray(arr)
        if a.dtype == np.float16:
            dt = KH_F16
        elif a.dtype == np.float32:
            dt = KH_F32
        else:
            raise TypeError(f"tensor {name}: dtype {a.dtype} is neither f32 nor f16")
        shape = (ctypes.c_int64 * max(1, a.ndim))(*a.shape)
        _check(self.lib, self.lib.kh_add_tensor(self.handle, name.encode(), dt, shape, a.ndim, _ptr(a), a.nbytes))

    @property
    def weight_bytes(self) -> int:
        return int(self.lib.kh_weight_bytes(self.handle))

    def check(self, plan: dict) -> None:
        js = plan_to_json(plan).encode()
        _check(self.lib, self.lib.kh_check(self.handle, js, len(js)))

    def runner(self, plan: dict) -> CudaPlanRunner:
        return CudaPlanRunner(self, plan)

    def fit_batch(self, build, batch: int):
        """The batch plan of the largest size up to `batch` that this backend accepts
        (src/plan/check.ts:129-138 tries 16, 8, 4)."""
        for b in (16, 8, 4):
            if b > batch:
                continue
            plan = build(b)
            try:
                self.check(plan)
                return plan
            except KhError:
                continue
        return None

    def prepare(self, work):
        return work()

    def call(self, start, read):
        return read(start())

    def bulk(self, runner: CudaPlanRunner, max_tokens: int, max_seqs: int, chunk_tokens: int = 65536) -> CudaBulk:
        return CudaBulk(runner, max_tokens, max_seqs, chunk_tokens)

    def info(self) -> dict:
        return json.loads(_string(self.lib.kh_info, self.handle))

    def inject_cuda_error(self, what: str) -> None:
        """Failure-path self-test: the next latching call reports a CUDA failure named `what`."""
        _check(self.lib, self.lib.kh_inject_cuda_error(self.handle, what.encode()))

    def selftest_wait_limit(self, limit_us: int) -> None:
        """Failure-path self-test: a bounded device wait gives up; raises the latched KhError."""
        _check(self.lib, self.lib.kh_selftest_wait_limit(self.handle, int(limit_us)))

    @property
    def stream(self) -> int:
        """cudaStream_t of every launch of this backend (for caller-side CUDA events)."""
        return int(self.lib.kh_ctx_stream(self.handle) or 0)

    def dispose(self) -> None:
        """Backend.dispose: frees the context with its plans and bulk handles still open."""
        if self.handle:
            self.lib.kh_destroy(self.handle)
            self.handle = None
            for r in list(self._runners):
                r._forget()

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass

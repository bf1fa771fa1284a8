"""kh_attention_f16_noalloc, the attention entry point that allocates no device memory, through the
C ABI. It is for callers that cannot allocate device memory while they serve (their memory is
budgeted up front, or a cudaMalloc would synchronize the device in the middle of their work).

Two calls in a row on caller-owned device buffers:
- sequences at a fixed stride with masked padding rows: equal to the plan path (kh_plan_create /
  kh_run over an attention op) on the same rows, and to the float64 reference;
- sequences of unequal lengths packed back to back (several of them sharing one 128-row tile,
  which is what the static sequence table is for): equal to a float64 reference per sequence.
After the calls the status query reports no pipeline wait that gave up; sizes beyond the limits
are refused with a status. Collected last, and also run alone in a fresh process."""
import numpy as np
import pytest

from kat_cases import attention_ref, prefix_mask
from test_gpu_attention import run_attention

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 4e-3, 1e-2  # f16 storage of q, k, v, P and ctx (as the other attention tests)


def packed_ref(qkv16, mask, lens, H, D, scale, window):
    """float64 attention of sequences packed back to back: row r of sequence s attends the kept
    rows of s within +-window of its own local position; masked query rows are zero."""
    hd = H * D
    x = np.nan_to_num(qkv16.astype(np.float64)).reshape(-1, 3, H, D)
    out = np.zeros((len(x), H, D))
    start = 0
    for n in lens:
        rows = np.arange(start, start + n)
        keep = mask[rows] > 0.5
        for h in range(H):
            q, k, v = x[rows, 0, h], x[rows, 1, h], x[rows, 2, h]
            s = q @ k.T * scale
            loc = np.arange(n)
            ok = keep[None, :] & ((np.abs(loc[:, None] - loc[None, :]) <= window) if window else True)
            s = np.where(ok, s, -np.inf)
            m = s.max(axis=1, keepdims=True)
            e = np.where(ok, np.exp(s - np.where(np.isfinite(m), m, 0)), 0.0)
            tot = e.sum(axis=1, keepdims=True)
            o = (e @ v) / np.where(tot > 0, tot, 1)
            out[rows, h] = np.where(keep[:, None], o, 0.0)
        start += n
    return out.reshape(-1)[: len(x) * hd]


def call_twice(qkv, mask, lens, H, D, scale, window, want, check_plan=None):
    import torch

    from kleinhirn_b200.backend import attention_f16_noalloc, attention_f16_noalloc_status
    hd = H * D
    dev = torch.device("cuda", 0)
    d_qkv = torch.from_numpy(qkv).to(dev)
    d_mask = torch.from_numpy(np.ascontiguousarray(mask, dtype=np.float32)).to(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    keep = np.repeat(mask > 0.5, hd)
    for call in range(2):  # the second call reuses the static table the first one wrote
        d_ctx = torch.full((len(mask) * hd,), float("nan"), dtype=torch.float16, device=dev)
        attention_f16_noalloc(d_qkv.data_ptr(), d_mask.data_ptr(), d_ctx.data_ptr(), lens, H, D, scale, window,
                              stream)
        attention_f16_noalloc_status(stream)
        got = d_ctx.cpu().numpy().astype(np.float64)
        assert np.all(got[~keep] == 0), f"call {call}: masked query rows must be exactly zero"
        for name, ref in (("float64", want), ("plan path", check_plan)):
            if ref is None:
                continue
            err = np.abs(got[keep] - ref[keep])
            tol = TOL_ABS + TOL_REL * np.abs(ref[keep])
            assert np.all(err <= tol), f"call {call} vs {name}: worst {err.max()}"


@pytest.mark.parametrize("D,H,L,lens,window", [
    (32, 12, 96, [96, 1, 90, 64, 30], 5),   # windowed, sequences shorter than their rows
    (64, 4, 300, [300, 129], 0),            # several key tiles per sequence
])
def test_noalloc_strided_matches_plan_path_and_float64(D, H, L, lens, window):
    B = len(lens)
    hd = H * D
    rng = np.random.default_rng(L + D)
    qkv = (rng.standard_normal(B * L * 3 * hd) * 1.5).astype(np.float16)
    mask = prefix_mask(L, lens)
    for r in range(B * L):
        if not mask[r]:
            qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
    scale = D ** -0.5
    plan = run_attention(qkv, mask, L, B, H, D, scale, window, B * L)
    want = attention_ref(qkv.astype(np.float32), mask, L, B, H, D, scale, window, B * L)
    call_twice(qkv, mask, [L] * B, H, D, scale, window, want, check_plan=plan)


@pytest.mark.parametrize("D,H,lens,window", [
    (32, 12, [96, 1, 90, 64, 30], 0),       # five sequences packed back to back in two tiles
    (32, 12, [96, 1, 90, 64, 30], 5),       # the same, windowed
    (64, 4, [7, 300, 129, 1, 40, 77], 0),   # sequences across tile boundaries, several key tiles
])
def test_noalloc_packed_unequal_lengths_float64(D, H, lens, window):
    hd = H * D
    T = int(sum(lens))
    rng = np.random.default_rng(T + D + window)
    qkv = (rng.standard_normal(T * 3 * hd) * 1.5).astype(np.float16)
    mask = np.ones(T, dtype=np.float32)
    # a few masked rows inside the packed sequences (their keys drop out, their rows are zero)
    for r in rng.choice(T, size=max(1, T // 40), replace=False):
        mask[r] = 0
        qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
    scale = D ** -0.5
    want = packed_ref(qkv, mask, lens, H, D, scale, window)
    call_twice(qkv, mask, lens, H, D, scale, window, want)


def test_noalloc_refuses_sizes_beyond_its_limits():
    from kleinhirn_b200.backend import KhError, attention_f16_noalloc
    with pytest.raises(KhError, match="n_seqs"):
        attention_f16_noalloc(16, 16, 16, [1] * 4097, 2, 32, 1.0)
    with pytest.raises(KhError, match="packed rows"):
        attention_f16_noalloc(16, 16, 16, [512] * 129, 2, 32, 1.0)
    with pytest.raises(KhError, match="sequence length"):
        attention_f16_noalloc(16, 16, 16, [20000], 2, 32, 1.0)
    with pytest.raises(KhError, match="head_dim"):
        attention_f16_noalloc(16, 16, 16, [8], 2, 48, 1.0)

"""kh_attention_f16_noalloc, the attention entry point that allocates no device memory, through the
C ABI: two calls in a row on caller-owned device buffers give what the plan path (kh_plan_create /
kh_run over an attention op) gives on the same rows, and sizes beyond its limits are refused with
a status. Collected last, and also run alone in a fresh process."""
import numpy as np
import pytest

from kat_cases import prefix_mask
from test_gpu_attention import run_attention

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D,H,L,lens,window", [
    (32, 12, 96, [96, 1, 90, 64, 30], 5),   # windowed, sequences shorter than their rows
    (64, 4, 300, [300, 129], 0),            # several key tiles per sequence
])
def test_noalloc_matches_the_plan_path(D, H, L, lens, window):
    import torch

    from kleinhirn_b200.backend import attention_f16_noalloc
    B = len(lens)
    hd = H * D
    rng = np.random.default_rng(L + D)
    qkv = (rng.standard_normal(B * L * 3 * hd) * 1.5).astype(np.float16)
    mask = prefix_mask(L, lens)
    for r in range(B * L):
        if not mask[r]:
            qkv[r * 3 * hd:(r + 1) * 3 * hd] = np.nan
    scale = D ** -0.5
    want = run_attention(qkv, mask, L, B, H, D, scale, window, B * L)

    dev = torch.device("cuda", 0)
    d_qkv = torch.from_numpy(qkv).to(dev)
    d_mask = torch.from_numpy(np.ascontiguousarray(mask, dtype=np.float32)).to(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    keep = np.repeat(mask > 0, hd)
    for call in range(2):  # the second call reuses the static table the first one wrote
        d_ctx = torch.full((B * L * hd,), float("nan"), dtype=torch.float16, device=dev)
        attention_f16_noalloc(d_qkv.data_ptr(), d_mask.data_ptr(), d_ctx.data_ptr(), [L] * B, H, D, scale,
                              window, stream)
        torch.cuda.synchronize(dev)
        got = d_ctx.cpu().numpy().astype(np.float64)
        assert np.all(got[~keep] == 0), f"call {call}: masked query rows must be exactly zero"
        err = np.abs(got[keep] - want[keep])
        tol = 4e-3 + 1e-2 * np.abs(want[keep])
        assert np.all(err <= tol), f"call {call}: worst {err.max()}"


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

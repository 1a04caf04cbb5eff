"""The allocation-free attention entry point against the workspace one, through the C ABI.

q3_attn_noalloc serves callers that cannot allocate device memory when they call in (a runtime
that owns a fixed device-memory budget, or code that must avoid the synchronisation cudaMalloc and
cudaFree can cause): its scratch is a static device array inside the library. This file sorts
last so that a run stopping at the first failure has run every other test before it; it passes
on its own in a fresh process as well.
"""
import numpy as np
import pytest

import gen_weights

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5  # the tolerance of the other attention parity tests


def _dev(torch, a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).cuda()
    return torch.from_numpy(a.copy()).cuda()


def test_attn_noalloc_matches_workspace_entry_point(q3lib):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    rng = np.random.default_rng(21)
    assert q3lib.lib().q3_attn_noalloc_max_scratch() == 64 * 256 * 4 + 256 + 64 * 8
    # Calls in a row on different shapes: each reuses (and must not be confused by) what the one
    # before left in the shared static scratch. The last two reach the static maximum: 64
    # splits (kv_len > 16128), at head_dim 128 and at 256, which fills the whole array.
    for kv_len, head_dim, n_kv, head in ((300, 128, 8, 0), (5000, 128, 8, 7), (16384, 128, 8, 3),
                                         (16500, 256, 2, 1)):
        q = _dev(torch, rng.standard_normal(head_dim).astype(np.float32))
        k = _dev(torch, gen_weights.f32_to_bf16_bits(
            rng.standard_normal((kv_len, n_kv * head_dim)).astype(np.float32)))
        v = _dev(torch, gen_weights.f32_to_bf16_bits(
            rng.standard_normal((kv_len, n_kv * head_dim)).astype(np.float32)))
        off = 2 * head * head_dim
        ws = torch.empty(q3lib.attn_workspace_size(head_dim, kv_len), dtype=torch.uint8,
                         device="cuda")
        want = torch.empty(head_dim, dtype=torch.float32, device="cuda")
        got = torch.empty(head_dim, dtype=torch.float32, device="cuda")
        q3lib.attn(want.data_ptr(), ws.data_ptr(), q.data_ptr(), k.data_ptr() + off,
                   v.data_ptr() + off, head_dim, n_kv, kv_len)
        q3lib.attn_noalloc(got.data_ptr(), q.data_ptr(), k.data_ptr() + off, v.data_ptr() + off,
                           head_dim, n_kv, kv_len)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL)


def test_attn_noalloc_rejects_bad_sizes(q3lib):
    with pytest.raises(q3lib.InvalidArgument):
        q3lib.attn_noalloc(0, 0, 0, 0, 512, 1, 16)  # head_dim above the static maximum

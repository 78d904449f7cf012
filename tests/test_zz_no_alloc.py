"""Decode attention through the entry point that allocates nothing.

Callers that cannot give the library a workspace (code running inside another
runtime's allocator callbacks, plugins whose host owns all device memory, paths
where a cudaMalloc would synchronise at a bad moment) use
dk_attention_batch_invariant_noalloc, which keeps its scratch in a fixed
library-owned device array.  These tests call it through the C ABI and check it
against the workspace entry point: two calls in a row with different shapes,
so the second call must not be disturbed by what the first left in the shared
scratch.  The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from oracle import ops as oracle

pytestmark = pytest.mark.gpu


def _noalloc(q, kc, vc, lens, max_len, scale=None):
    import torch

    from detkernels_b200 import _lib

    R, H, D = q.shape
    n_seq, Hkv, cap, _ = kc.shape
    out = torch.empty_like(q)
    scale = 1.0 / (D ** 0.5) if scale is None else scale
    lib = _lib.load()
    rc = lib.dk_attention_batch_invariant_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1),
        kc.stride(2), n_seq, cap, out.data_ptr(), out.stride(0), out.stride(1), lens.data_ptr(), 0, None, 0,
        R, H, Hkv, D, int(max_len), float(scale), _lib.dtype_code(q.dtype), _lib.stream_ptr(q.device))
    _lib.check(rc, "dk_attention_batch_invariant_noalloc")
    return out


def _case(dev, seed, B, H, Hkv, S, D):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, H, D, device=dev, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    lens = torch.randint(1, S + 1, (B,), device=dev, generator=g).to(torch.int32)
    lens[0] = S
    return q, kc, vc, lens


def test_noalloc_matches_workspace_entry_on_two_calls(dev):
    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels.attention import attention_decode

    cases = [(11, 6, 32, 8, 2000, 128), (12, 9, 16, 16, 700, 64)]
    for seed, B, H, Hkv, S, D in cases:
        q, kc, vc, lens = _case(dev, seed, B, H, Hkv, S, D)
        got = _noalloc(q, kc, vc, lens, S)
        want = attention_decode(q, kc, vc, lens, max_kv_len=S)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (seed, B, H, Hkv, S, D)
        ref = oracle.attention(q.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                               kv_lens=lens.cpu().numpy())
        np.testing.assert_allclose(got.float().cpu().numpy(), ref, rtol=2 ** -6, atol=2 ** -6)
    code, detail = _lib.device_status(torch.cuda.current_device())
    assert code == 0, (code, detail)


def test_noalloc_rejects_calls_beyond_its_scratch(dev):
    import torch

    from detkernels_b200 import _lib

    lib = _lib.load()
    limit = lib.dk_attention_noalloc_scratch_limit()
    assert limit == 32 << 20
    # 4096 rows x 8 kv heads x 32 splits x 4 rows x 130 floats is far beyond 32 MiB; the cache
    # really holds the 8192 tokens the call describes, so even a call that got past the size
    # check would read only allocated memory
    q = torch.zeros(4096, 32, 128, device=dev, dtype=torch.bfloat16)
    kc = torch.zeros(1, 8, 8192, 128, device=dev, dtype=torch.bfloat16)
    lens = torch.ones(4096, device=dev, dtype=torch.int32)
    out = torch.empty_like(q)
    rc = lib.dk_attention_batch_invariant_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), kc.data_ptr(), kc.stride(0), kc.stride(1),
        kc.stride(2), 1, 8192, out.data_ptr(), out.stride(0), out.stride(1), lens.data_ptr(), 0, None, 0,
        4096, 32, 8, 128, 8192, ctypes.c_float(0.088), _lib.DK_BF16, _lib.stream_ptr(q.device))
    assert rc == _lib.DK_ERR_WORKSPACE
    assert "built-in scratch" in _lib.last_error()


def test_noalloc_clears_stale_counters_left_in_its_scratch(dev):
    """A call that stopped early can leave non-zero arrival counters in the shared scratch.
    Fill the start of the scratch with garbage through a test hook that is not part of the
    public header, then check the next call still gives the workspace entry point's bits."""
    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels.attention import attention_decode

    lib = _lib.load()
    fill = lib.dk_noalloc_scratch_fill_for_test
    fill.restype = ctypes.c_int
    fill.argtypes = [ctypes.c_int, ctypes.c_size_t]
    for seed, B, H, Hkv, S, D in [(21, 5, 32, 8, 3000, 128), (22, 7, 16, 16, 900, 64)]:
        q, kc, vc, lens = _case(dev, seed, B, H, Hkv, S, D)
        want = attention_decode(q, kc, vc, lens, max_kv_len=S)
        torch.cuda.synchronize()
        _lib.check(fill(0x5A, 1 << 16), "dk_noalloc_scratch_fill_for_test")
        got = _noalloc(q, kc, vc, lens, S)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (seed, B, H, Hkv, S, D)

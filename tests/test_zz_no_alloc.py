"""The allocation-free linear cross-entropy forward (gptb200_lce_fwd_noalloc).

Some callers cannot allocate device memory or hand the library a workspace:
an XLA custom-call handler only gets buffers from XLA's own allocator, and code
that records a CUDA graph may not call cudaMalloc. This entry point keeps its
scratch in a fixed device array inside libgptb200.so instead. The test calls
it through the C ABI twice in a row (the array is shared and keeps the last
call's contents) and checks both results against the workspace entry point,
gptb200_lce_fwd, with the tolerance of tests/test_lce.py; sizes beyond the
array must be rejected before anything runs.
"""

import ctypes

import pytest
import torch

from rig_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(dev, n, d, v, sv, seed):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(n, d, generator=g).bfloat16().to(dev)
    e = (0.02 * torch.randn(v, d, generator=g)).bfloat16().to(dev)
    t = torch.randint(0, sv, (n,), generator=g, dtype=torch.int32)
    t[7] = -1  # one invalid target: +inf loss on both paths
    return h, e, t.to(dev)


def _with_workspace(lib, h, e, t, sv, stream):
    n, d = h.shape
    v = e.shape[0]
    ws = torch.empty(lib.gptb200_lce_fwd_workspace_size(n, v), dtype=torch.uint8, device=h.device)
    losses = torch.empty(n, device=h.device)
    lse = torch.empty(n, device=h.device)
    mean = torch.empty(1, device=h.device)
    _lib.check(lib.gptb200_lce_fwd(_ptr(h), _ptr(e), _ptr(t), n, d, v, sv, _ptr(losses), _ptr(lse),
                                   _ptr(mean), _ptr(ws), stream), "gptb200_lce_fwd")
    return losses, lse, mean


def _no_alloc(lib, h, e, t, sv, stream):
    n, d = h.shape
    v = e.shape[0]
    losses = torch.full((n,), float("nan"), device=h.device)
    lse = torch.full((n,), float("nan"), device=h.device)
    mean = torch.full((1,), float("nan"), device=h.device)
    _lib.check(lib.gptb200_lce_fwd_noalloc(_ptr(h), _ptr(e), _ptr(t), n, d, v, sv, _ptr(losses),
                                           _ptr(lse), _ptr(mean), stream),
               "gptb200_lce_fwd_noalloc")
    return losses, lse, mean


def test_no_alloc_matches_workspace_entry_point_twice(cuda):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cases = [(2048, 256, 50304, 50257, 11), (1000, 128, 5000, 4990, 12)]
    for n, d, v, sv, seed in cases:  # two calls in a row, different shapes
        h, e, t = _case(cuda, n, d, v, sv, seed)
        want = _with_workspace(lib, h, e, t, sv, stream)
        got = _no_alloc(lib, h, e, t, sv, stream)
        torch.cuda.synchronize()
        assert ops.device_error() == 0  # no GEMM wait ran out inside either call
        for a, b in zip(got[:2], want[:2]):
            ok = torch.isfinite(b)
            assert torch.equal(torch.isfinite(a), ok)
            assert torch.allclose(a[ok], b[ok], rtol=1e-4, atol=2e-4)
        assert torch.isinf(got[0][7]) and torch.isinf(got[2]).all()


def test_no_alloc_rejects_sizes_beyond_its_scratch(cuda):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    h, e, t = _case(cuda, 8192, 64, 50304, 50304, 3)  # 8192 x 197 tiles > 2^20 partials
    out = torch.empty(8192, device=cuda)
    status = lib.gptb200_lce_fwd_noalloc(_ptr(h), _ptr(e), _ptr(t), 8192, 64, 50304, 50304,
                                         _ptr(out), _ptr(out), None, stream)
    assert status == 6  # GPTB200_ETOOLARGE
    assert b"scratch" in lib.gptb200_status_string(status)

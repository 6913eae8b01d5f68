"""klg_fwd_noalloc -- the forward for callers that cannot allocate device memory
(for instance a runtime that has reserved all device memory for its own
allocator, or a latency-critical loop that must not pay cudaMalloc's
device-wide synchronisation) -- gives the same results as klg_fwd.

Called through the C-ABI on two problems in a row, so the second call also
shows that what the first call left in the shared scratch array does not leak
into its results.  Collected last (file name) so a failure here does not hide
the other tests' results.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.gpu_helpers import LOSS_RTOL

pytestmark = pytest.mark.gpu

_vp = ctypes.c_void_p


def _p(t):
    return _vp(t.data_ptr()) if t is not None else _vp(0)


def _problem(N, H, V, seed, T):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda:0")
    hs = torch.randn(N, H, generator=g).to(dev, torch.bfloat16)
    ht = (torch.randn(N, H, generator=g) * 2).to(dev, torch.bfloat16)
    w = (torch.randn(V, H, generator=g) * 0.02).to(dev, torch.bfloat16)
    m = (torch.rand(N, generator=g) < 0.5).to(torch.uint8).to(dev)
    return hs, ht, w, m, T


def _outputs(N, dev):
    return (torch.empty(1, device=dev), torch.empty((), device=dev), torch.empty(2, N, device=dev),
            torch.empty(N, device=dev))


def _run_both(hs, ht, w, m, T):
    from orthrus_training_test_b200 import _lib
    L = _lib.lib()
    N, H = hs.shape
    V = w.shape[0]
    dev = hs.device
    stream = _vp(torch.cuda.current_stream(dev).cuda_stream)
    # existing entry point with a caller-allocated workspace
    ws_bytes = L.klg_fwd_workspace_bytes(N, V)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    c0, l0, lse0, kl0 = _outputs(N, dev)
    _lib.check("klg_fwd", L.klg_fwd(_p(hs), _p(ht), _p(w), _p(m), N, H, V, 1.0 / T, 0, _p(c0), _p(l0), _p(lse0),
                                    _p(kl0), _p(ws), ws_bytes, stream))
    # allocation-free entry point
    c1, l1, lse1, kl1 = _outputs(N, dev)
    _lib.check("klg_fwd_noalloc", L.klg_fwd_noalloc(_p(hs), _p(ht), _p(w), _p(m), N, H, V, 1.0 / T, 0, _p(c1),
                                                    _p(l1), _p(lse1), _p(kl1), stream))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return (c0, l0, lse0, kl0), (c1, l1, lse1, kl1)


def test_noalloc_forward_matches_workspace_forward_twice():
    for (N, H, V, seed, T) in [(1000, 576, 3000, 1, 1.0), (333, 128, 1500, 2, 2.0)]:
        ref, ours = _run_both(*_problem(N, H, V, seed, T))
        c0, l0, lse0, kl0 = (x.cpu().double().numpy() for x in ref)
        c1, l1, lse1, kl1 = (x.cpu().double().numpy() for x in ours)
        assert c0 == c1
        assert abs(float(l1) - float(l0)) <= LOSS_RTOL * abs(float(l0))
        np.testing.assert_allclose(lse1, lse0, rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(kl1, kl0, rtol=1e-5, atol=1e-7)


def test_noalloc_rejects_problems_beyond_its_scratch():
    from orthrus_training_test_b200 import _lib
    L = _lib.lib()
    cap = L.klg_fwd_noalloc_max_floats()
    assert cap == 4 << 20
    N, H, V = 1 << 20, 64, 1 << 16          # needs far more than the fixed scratch
    hs = torch.empty(8, dtype=torch.bfloat16, device="cuda:0")
    out = torch.empty(4, device="cuda:0")
    rc = L.klg_fwd_noalloc(_p(hs), _p(hs), _p(hs), _p(hs), N, H, V, 1.0, 0, _p(out), _p(out), _p(out), None,
                           _vp(torch.cuda.current_stream().cuda_stream))
    assert rc == _lib.KLG_ERR_WORKSPACE
    assert "klg_fwd_noalloc" in _lib.last_error()

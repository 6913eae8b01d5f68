"""Failure detection on the GPU without a fault.

Every pipeline wait in the kernels is bounded: past the bound it sets a bit in the
device status word and the kernel ends early instead of hanging.  The self-test hook
runs that same bounded wait on an mbarrier nothing completes; the test checks the bit,
the time it took, and that the context still computes correct losses afterwards.
"""
import ctypes
import time

import pytest
import torch

from oracle import klgemm_oracle as O
from tests.gpu_helpers import LOSS_RTOL

pytestmark = pytest.mark.gpu

KLG_STATUS_SELFTEST = 0x100


def test_bounded_wait_reports_and_context_survives():
    from orthrus_training_test_b200 import _lib, ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    torch.zeros(1, device=dev)                      # context up before timing
    assert _lib.device_status(reset=True) == 0
    t0 = time.perf_counter()
    _lib.call("klg_selftest_wait_timeout", ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    status = _lib.device_status(reset=True)
    assert status == KLG_STATUS_SELFTEST, hex(status)
    assert 0.2 < waited < 30.0, waited             # the bound is ~2^31 cycles (~1 s)

    # the context is intact: a loss right after matches the oracle and sets no status bit
    g = torch.Generator().manual_seed(3)
    h_s = torch.randn(300, 128, generator=g)
    h_t = torch.randn(300, 128, generator=g)
    W = torch.randn(700, 128, generator=g) * 0.1
    mask = torch.rand(300, generator=g) < 0.6
    loss = ops.kl_gemm_loss(h_s.to(dev).to(torch.bfloat16), h_t.to(dev).to(torch.bfloat16),
                            W.to(dev).to(torch.bfloat16), mask.to(dev))
    bf = lambda x: x.to(torch.bfloat16).float().numpy()
    ref = O.aligned_kl_loss_np(bf(h_s), bf(h_t), bf(W), mask.numpy(), 1.0)[0]
    assert abs(float(loss) - ref) <= LOSS_RTOL * abs(ref)
    assert _lib.device_status(reset=True) == 0

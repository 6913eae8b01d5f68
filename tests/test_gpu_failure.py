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


def test_attention_split_timeout_reports_and_cluster_exits():
    """A decode call whose AR key range is split over a thread-block cluster: one split is
    starved of its loads (test hook), its operand wait runs out its bound, and every CTA of
    the cluster still meets at the (unbounded) cluster barriers and exits -- the call ends
    with a timeout status instead of hanging, and the next call is correct."""
    import math

    from orthrus_training_test_b200 import _lib
    from orthrus_training_test_b200.attention import block_attention
    from orthrus_training_test_b200.ops import _ptr, _stream

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    B, H, Hkv, K, AL, D = 1, 9, 3, 32, 2048, 64
    splits = _lib.lib().klg_block_attn_splits(B, H, Hkv, K, K, AL, D)
    assert splits >= 2, splits
    g = torch.Generator().manual_seed(11)
    q = torch.randn(B, H, K, D, generator=g).to(torch.bfloat16).to(dev)
    ks, vs = (torch.randn(B, Hkv, K, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(2))
    ka, va = (torch.randn(B, Hkv, AL, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(2))
    lim = torch.full((B, K), AL - 1, dtype=torch.int32, device=dev)
    out = torch.empty(B, H, K, D, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(256, dtype=torch.uint8, device=dev)
    assert _lib.device_status(reset=True) == 0
    t0 = time.perf_counter()
    _lib.call("klg_selftest_attn_split_stall", _ptr(q), _ptr(ks), _ptr(vs), _ptr(ka), _ptr(va), AL, _ptr(lim), B, H,
              Hkv, K, K, AL, D, 1.0 / math.sqrt(D), _ptr(out), None, _ptr(ws), 256, splits // 2, _stream(dev))
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    status = _lib.device_status(reset=True)
    assert status & 0x7, hex(status)                # a pipeline wait gave up and said so
    assert 0.2 < waited < 60.0, waited

    # the context is intact: the same call without the hook matches the oracle
    o = block_attention(q, ks, vs, ka, va, lim, K)
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    ro, _ = O.block_attention_np(q.float().cpu().numpy(), ks.float().cpu().numpy(), vs.float().cpu().numpy(),
                                 ka.float().cpu().numpy(), va.float().cpu().numpy(), lim.cpu().numpy(), K)
    assert float((o.float().cpu() - torch.tensor(ro)).abs().max()) <= 3e-2


def test_exchange_wait_on_a_missing_rank_times_out():
    """The in-step dW exchange waits for every rank's epoch flag; a rank that never arrives
    (here: an epoch nobody publishes, on one GPU, through the test hook) makes the wait give up
    after its bound with KLG_STATUS_TIMEOUT_PEER instead of hanging, and the context stays usable."""
    from orthrus_training_test_b200 import _lib, ops

    KLG_STATUS_TIMEOUT_PEER = 0x10
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    V, H = 1000, 128
    nbytes = int(_lib.lib().klg_xr_buffer_bytes(V, H, 2))
    assert nbytes > 0
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    assert _lib.device_status(reset=True) == 0
    t0 = time.perf_counter()
    _lib.call("klg_selftest_xr_timeout", ops._ptr(buf), V, H, ops._stream(dev))
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    status = _lib.device_status(reset=True)
    assert status == KLG_STATUS_TIMEOUT_PEER, hex(status)
    assert 0.2 < waited < 30.0, waited
    x = torch.ones(1 << 20, device=dev)
    assert float(x.sum()) == float(1 << 20)         # the context still runs kernels
    assert _lib.device_status(reset=True) == 0

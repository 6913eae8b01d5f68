"""Fused final-RMSNorm prologue (pre-norm inputs) against the oracle and the reference.

The norm kernel's bf16 rows equal transformers' LlamaRMSNorm (the reference's final norm,
model.py:493) to one bf16 ulp on the golden fixture (>= 99.9 % bit-exact: the fp32 mean of
squares is summed in another order); rstd to 2e-6 relative, and the rows bit-exact given
the device's rstd; the backward to 1e-5 of the largest entry against float64.  Through the loss: the golden loss (reference
compute_kl_loss on normed fp32 rows) to 1e-3 relative and its pre-norm gradient to the
gradient tolerances of every GPU test (the GEMMs run in bf16).
"""
import numpy as np
import pytest
import torch

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN
from tests.gpu_helpers import GRAD_COS, GRAD_MAX_REL, LOSS_RTOL

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda:0")


def _ulps(a, b):
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64) >> 16
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64) >> 16
    return np.abs(ia - ib)


def _grad_ok(ours, ref, what):
    err, cos = O.grad_metrics(np.asarray(ours, np.float64), np.asarray(ref, np.float64))
    assert err <= GRAD_MAX_REL and cos >= GRAD_COS, f"{what}: max-rel {err:.3e} cos {cos:.6f}"


def test_norm_matches_reference_golden():
    from orthrus_training_test_b200 import _lib, ops
    g = dict(np.load(GOLDEN / "norm_bf16.npz"))
    x = torch.tensor(g["x"]).to(torch.bfloat16).to(_dev())
    y, r = ops.rmsnorm_rows(x, torch.tensor(g["gamma"]), float(g["eps"]))
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    d = _ulps(y.float().cpu().numpy(), g["y"])
    assert d.max() <= 1 and np.mean(d == 0) >= 0.999, (d.max(), np.mean(d == 0))


@pytest.mark.parametrize("N,H,dtype", [(1, 8, torch.bfloat16), (300, 576, torch.bfloat16), (4096, 2048, torch.bfloat16),
                                       (1000, 1024, torch.float32), (77, 264, torch.float32)])
def test_norm_rows_and_backward_match_oracle(N, H, dtype):
    from orthrus_training_test_b200 import ops
    gen = torch.Generator().manual_seed(N + H)
    x = (torch.randn(N, H, generator=gen) * 3.0).to(dtype)
    gam = (1.0 + 0.3 * torch.randn(H, generator=gen)).to(torch.bfloat16).float()
    dy = torch.randn(N, H, generator=gen)
    y, r = ops.rmsnorm_rows(x.to(_dev()), gam, 1e-5)
    dx = ops.rmsnorm_rows_backward(x.to(_dev()), gam, r, dy.to(_dev()))
    torch.cuda.synchronize()
    bf = dtype == torch.bfloat16
    _, ro = O.rmsnorm_np(x.float().numpy(), gam.numpy(), 1e-5, bf16_input=bf)
    np.testing.assert_allclose(r.cpu().numpy(), ro, rtol=2e-6)
    # given the device's r, the rows are bit-exact (the roundings and products are the same)
    yo, _ = O.rmsnorm_np(x.float().numpy(), gam.numpy(), 1e-5, bf16_input=bf, r=r.cpu().numpy())
    if not bf:
        yo = O._bf16_round_np(yo)
    np.testing.assert_array_equal(y.float().cpu().numpy(), yo)
    dxo = O.rmsnorm_backward_np(x.float().numpy(), gam.numpy(), r.cpu().numpy(), dy.numpy())
    err = np.abs(dx.cpu().numpy() - dxo).max() / np.abs(dxo).max()
    assert err <= 1e-5, err


def test_prenorm_loss_matches_reference_golden():
    from orthrus_training_test_b200 import prenorm_kl_loss
    g = dict(np.load(GOLDEN / "norm_loss.npz"))
    xs = torch.tensor(g["h_s"]).to(_dev()).requires_grad_(True)
    loss = prenorm_kl_loss(xs, torch.tensor(g["h_t"]).to(_dev()), torch.tensor(g["gamma"]),
                           torch.tensor(g["weight"]).to(_dev()), torch.tensor(g["mask"]).to(_dev()), 1.0,
                           float(g["eps"]))
    loss.backward()
    ref = float(g["loss"])
    assert abs(float(loss) - ref) <= LOSS_RTOL * abs(ref)
    _grad_ok(xs.grad.cpu().numpy(), g["grad_h_s"], "dx_s (pre-norm)")


def test_prenorm_matches_oracle_on_device_rows():
    """bf16 pre-norm rows at a trainer-like size: the loss and dx against the float64 oracle
    run on the device's own normed rows (so only the loss arithmetic is compared)."""
    from orthrus_training_test_b200 import ops, prenorm_kl_loss
    gen = torch.Generator().manual_seed(5)
    N, H, V, T = 2048, 576, 8192, 1.0
    xs = (torch.randn(N, H, generator=gen) * 3.0).to(torch.bfloat16)
    xt = (torch.randn(N, H, generator=gen) * 3.0).to(torch.bfloat16)
    gam = (1.0 + 0.3 * torch.randn(H, generator=gen)).to(torch.bfloat16)
    W = (torch.randn(V, H, generator=gen) * 0.05).to(torch.bfloat16)
    mask = torch.rand(N, generator=gen) < 0.6
    xsd = xs.to(_dev()).requires_grad_(True)
    loss = prenorm_kl_loss(xsd, xt.to(_dev()), gam, W.to(_dev()), mask.to(_dev()), T)
    loss.backward()
    ys, rs = ops.rmsnorm_rows(xs.to(_dev()), gam)
    yt, _ = ops.rmsnorm_rows(xt.to(_dev()), gam)
    ref_loss, dh, _, _, _, _ = O.aligned_kl_loss_np(ys.float().cpu().numpy(), yt.float().cpu().numpy(),
                                                     W.float().numpy(), mask.numpy(), T)
    assert abs(float(loss) - ref_loss) <= LOSS_RTOL * abs(ref_loss)
    dxo = O.rmsnorm_backward_np(xs.float().numpy(), gam.float().numpy(), rs.cpu().numpy(), dh)
    _grad_ok(xsd.grad.float().cpu().numpy(), dxo, "dx_s")


def test_compute_kl_loss_with_norm_weight_equals_prenormed_call():
    from orthrus_training_test_b200 import compute_kl_loss, ops
    gen = torch.Generator().manual_seed(8)
    B, Bb, K, L, H, V = 2, 3, 6, 20, 64, 203
    diff = (torch.randn(B, Bb * K, H, generator=gen) * 2.0).to(_dev())
    ar = (torch.randn(B, L, H, generator=gen) * 2.0).to(_dev())
    anchors = torch.tensor([[0, 9, 17], [3, 15, 19]], device=_dev())
    tgt = torch.randint(1, 50, (B, Bb * K), generator=gen).to(_dev())
    gam = (1.0 + 0.2 * torch.randn(H, generator=gen)).to(_dev())
    head = torch.nn.Linear(H, V, bias=False).to(_dev())
    torch.nn.init.normal_(head.weight, std=0.05, generator=None)
    d1 = diff.clone().requires_grad_(True)
    l1 = compute_kl_loss(d1, ar, head, anchors, K, tgt, 0, norm_weight=gam)
    l1.backward()
    # the same through an explicit norm: the kernel's bf16 normed rows, then the plain op on bf16
    # operands (the fused norm's loss runs on bf16 rows and the bf16-rounded head; fp32 operands
    # would take the fp32-faithful path instead)
    d2 = diff.clone().requires_grad_(True)
    y = ops.rmsnorm_rows(d2.reshape(-1, H), gam)[0].reshape(d2.shape)
    ya = ops.rmsnorm_rows(ar.reshape(-1, H), gam)[0].reshape(ar.shape)
    head16 = torch.nn.Linear(H, V, bias=False).to(_dev(), torch.bfloat16)
    with torch.no_grad():
        head16.weight.copy_(head.weight)
    l2 = compute_kl_loss(y, ya, head16, anchors, K, tgt, 0)
    assert abs(float(l1) - float(l2)) <= 1e-6 * abs(float(l2))
    assert d1.grad is not None and torch.isfinite(d1.grad).all()

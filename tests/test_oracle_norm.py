"""Pin the final-RMSNorm oracle against the reference's own norm and loss.

Fixtures from ``tests/golden/make_golden_norm.py``: the backbone's final norm
(``model.py:493``, transformers ``LlamaRMSNorm``) on bf16 rows, and
``train.compute_kl_loss`` (``train.py:142-195``) on fp32 rows through that norm, with the
gradient of the pre-norm student rows.
"""
import numpy as np

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def bf16_ulps(a, b):
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64) >> 16
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64) >> 16
    return np.abs(ia - ib)


def test_norm_bf16_matches_reference():
    g = load("norm_bf16")
    y, r = O.rmsnorm_np(g["x"], g["gamma"], float(g["eps"]), bf16_input=True)
    d = bf16_ulps(y, g["y"])
    assert d.max() <= 1 and np.mean(d == 0) >= 0.999, (d.max(), np.mean(d == 0))
    assert np.all(np.isfinite(r)) and r.shape == (g["x"].shape[0],)


def test_prenorm_loss_and_grad_match_reference():
    g = load("norm_loss")
    loss, dx = O.prenorm_kl_loss_np(g["h_s"], g["h_t"], g["gamma"], g["weight"], g["mask"], 1.0, float(g["eps"]))
    assert abs(loss - float(g["loss"])) <= 1e-5 * abs(float(g["loss"]))
    np.testing.assert_allclose(dx, g["grad_h_s"], rtol=1e-3, atol=1e-6 * np.abs(g["grad_h_s"]).max())


def test_norm_backward_matches_finite_differences():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(5, 64)) * 2.0
    gam = 1.0 + 0.3 * rng.normal(size=64)
    dy = rng.normal(size=(5, 64))

    def f(xx):
        var = np.mean(xx ** 2, axis=-1, keepdims=True)
        return (gam * xx / np.sqrt(var + 1e-5) * dy).sum()

    r = 1.0 / np.sqrt(np.mean(x ** 2, axis=-1) + 1e-5)
    dx = O.rmsnorm_backward_np(x, gam, r, dy)
    num = np.zeros_like(x)
    h = 1e-6
    for i in range(x.shape[0]):
        for j in range(x.shape[1]):
            e = np.zeros_like(x)
            e[i, j] = h
            num[i, j] = (f(x + e) - f(x - e)) / (2 * h)
    np.testing.assert_allclose(dx, num, rtol=1e-5, atol=1e-7)

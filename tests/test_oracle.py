"""Pin the oracle against golden vectors produced by the reference itself.

The fixtures in ``tests/golden`` come from running the reference's
``train.compute_kl_loss`` (train.py:142-195); ``tests/golden/make_golden.py``
is the generator.  Tolerances here are fp32-vs-fp32 (the oracle and the
reference run the same arithmetic).
"""
import numpy as np
import pytest
import torch

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN, golden_cases


def load(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


@pytest.mark.parametrize("name", golden_cases())
def test_reference_ops_match_golden(name):
    g = load(name)
    diff = torch.tensor(g["diff_hidden"], requires_grad=True)
    W = torch.tensor(g["weight"], requires_grad=True)
    with O.fp32_strict():
        loss = O.kl_loss_reference_ops(diff, torch.tensor(g["ar_hidden"]), W,
                                       torch.tensor(g["anchor_positions"]), int(g["K"]),
                                       torch.tensor(g["target_ids"]), int(g["pad"]),
                                       temperature=float(g["temperature"]))
        assert abs(loss.item() - float(g["loss"])) <= 1e-6 * max(1.0, abs(float(g["loss"])))
        if loss.grad_fn is not None:
            loss.backward()
            np.testing.assert_allclose(diff.grad.numpy(), g["grad_diff_hidden"], rtol=1e-4, atol=1e-7)
            np.testing.assert_allclose(W.grad.numpy(), g["grad_weight"], rtol=1e-4, atol=1e-7)


@pytest.mark.parametrize("name", golden_cases())
def test_select_rows_matches_reference_gather(name):
    """Row selection (train.py:124-139, 156-164) reproduces the aligned rows."""
    g = load(name)
    h_s, h_t, valid, _, _ = O.select_rows_np(g["diff_hidden"], g["ar_hidden"], g["anchor_positions"],
                                             int(g["K"]), g["target_ids"], int(g["pad"]))
    if "h_s" in g:
        np.testing.assert_array_equal(h_s, g["h_s"])
        np.testing.assert_array_equal(h_t, g["h_t"])
        np.testing.assert_array_equal(valid, g["mask"])
    # gradient of the loss lands only on the selected student rows
    gd = g["grad_diff_hidden"]
    B, Ld, _ = gd.shape
    dp, bi, _ = O.kl_indices(*g["anchor_positions"].shape, int(g["K"]))
    sel = np.zeros((B, Ld), bool)
    sel[bi, dp] = True
    assert np.all(gd[~sel] == 0)


@pytest.mark.parametrize("name", golden_cases())
def test_numpy_closed_form_matches_golden(name):
    g = load(name)
    h_s, h_t, valid, dp, _ = O.select_rows_np(g["diff_hidden"], g["ar_hidden"], g["anchor_positions"],
                                              int(g["K"]), g["target_ids"], int(g["pad"]))
    loss, dH, dW, *_ = O.aligned_kl_loss_np(h_s, h_t, g["weight"], valid, float(g["temperature"]))
    assert abs(loss - float(g["loss"])) <= 2e-6 * max(1.0, abs(float(g["loss"])))
    B = g["anchor_positions"].shape[0]
    gsel = g["grad_diff_hidden"][np.arange(B)[:, None], dp].reshape(dH.shape)
    np.testing.assert_allclose(dH, gsel, rtol=1e-4, atol=1e-8)
    np.testing.assert_allclose(dW, g["grad_weight"], rtol=1e-4, atol=1e-8)


@pytest.mark.parametrize("name", [n for n in golden_cases() if n.startswith("aligned")])
def test_aligned_torch_matches_golden(name):
    g = load(name)
    loss, dh, dw = O.aligned_kl_torch_with_grads(torch.tensor(g["h_s"]), torch.tensor(g["h_t"]),
                                                 torch.tensor(g["weight"]), torch.tensor(g["mask"]),
                                                 float(g["temperature"]))
    assert abs(loss.item() - float(g["loss"])) <= 1e-6 * max(1.0, abs(float(g["loss"])))
    np.testing.assert_allclose(dw.numpy(), g["grad_weight"], rtol=1e-4, atol=1e-7)


@pytest.mark.parametrize("name", [n for n in golden_cases() if n.startswith("aligned")])
def test_partial_merge_equals_full(name):
    """Splitting the vocab into ranges and merging partial records is exact."""
    g = load(name)
    W = g["weight"]
    T = float(g["temperature"])
    cuts = [0, 37, 128, 129, W.shape[0]]
    parts = [O.partial_stats_np(g["h_s"], g["h_t"], W[a:b], T) for a, b in zip(cuts[:-1], cuts[1:])]
    merged = O.merge_partials_np(parts)
    loss, row_kl, ls, lt = O.finalize_np(merged, g["mask"])
    assert abs(loss - float(g["loss"])) <= 2e-6 * max(1.0, float(g["loss"]))
    n = g["mask"].sum()
    dH = 0
    dW = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        dh, dw = O.range_grads_np(g["h_s"], g["h_t"], W[a:b], ls, lt, g["mask"], n, T)
        dH = dH + dh
        dW.append(dw)
    np.testing.assert_allclose(np.concatenate(dW), g["grad_weight"], rtol=1e-4, atol=1e-8)


def test_all_masked_is_zero():
    g = load("all_masked")
    assert float(g["loss"]) == 0.0
    assert not g["grad_weight"].any()


def test_make_problem_shapes():
    p = O.make_problem("c5", n_rows=12288 - 37)
    assert p["h_s"].shape == (12288 - 37, 576) and p["h_s"].dtype == torch.bfloat16
    assert p["T"] == 2.0
    assert not p["mask"][:8].any()
    frac = p["mask"].float().mean().item()
    assert 0.15 < frac < 0.35

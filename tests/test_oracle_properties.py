"""Properties of the oracle beyond the reference's golden fixtures, on seeded random problems
(no GPU): its float64 closed form, the reference's fp32 op sequence and the vocab-range
partial / merge maths agree with each other, and the closed-form gradients agree with finite
differences of the loss.  The golden fixtures (tests/test_oracle.py) pin the oracle to the
reference at five points; these checks cover the shapes, temperatures and masks in between."""
import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import klgemm_oracle as O

problems = st.tuples(st.integers(1, 24), st.sampled_from([8, 16, 64]), st.integers(1, 300),
                     st.sampled_from([0.5, 1.0, 2.0]), st.floats(0.0, 1.0), st.integers(0, 2 ** 31 - 1))


def _problem(N, H, V, p_valid, seed, t_scale=1.0):
    rng = np.random.default_rng(seed)
    h_s = rng.standard_normal((N, H))
    h_t = rng.standard_normal((N, H)) * t_scale
    W = rng.standard_normal((V, H)) * 0.3
    mask = rng.random(N) < p_valid
    return h_s, h_t, W, mask


@settings(max_examples=40, deadline=None, derandomize=True)
@given(problems)
def test_closed_form_matches_reference_op_sequence(prob):
    """float64 closed form against the reference's fp32 op order (train.py:188-210) with
    autograd gradients: fp32 agreement."""
    N, H, V, T, p_valid, seed = prob
    h_s, h_t, W, mask = _problem(N, H, V, p_valid, seed)
    loss, dH, dW, *_ = O.aligned_kl_loss_np(h_s, h_t, W, mask, T)
    tl, tdh, tdw = O.aligned_kl_torch_with_grads(torch.tensor(h_s), torch.tensor(h_t), torch.tensor(W),
                                                 torch.tensor(mask), T)
    if not mask.any():
        assert loss == 0.0 and float(tl) == 0.0 and not dH.any() and not dW.any()
        return
    assert abs(float(tl) - loss) <= 1e-5 * max(1.0, abs(loss))
    scale = max(np.abs(dH).max(), np.abs(dW).max(), 1e-12)
    assert np.abs(tdh.double().numpy() - dH).max() <= 1e-4 * scale
    assert np.abs(tdw.double().numpy() - dW).max() <= 1e-4 * scale


@settings(max_examples=40, deadline=None, derandomize=True)
@given(problems, st.lists(st.floats(0.0, 1.0), min_size=1, max_size=4))
def test_vocab_ranges_merge_to_the_whole(prob, cuts):
    """Any split of the vocabulary into ranges, merged online, gives the full-vocab loss,
    log-sum-exps and gradients (float64, to rounding)."""
    N, H, V, T, p_valid, seed = prob
    h_s, h_t, W, mask = _problem(N, H, V, p_valid, seed, t_scale=2.0)
    if not mask.any():
        mask[0] = True
    loss, dH, dW, row_kl, lse_s, lse_t = O.aligned_kl_loss_np(h_s, h_t, W, mask, T)
    edges = sorted({0, V, *[int(c * V) for c in cuts]})
    parts = [O.partial_stats_np(h_s, h_t, W[a:b], T) for a, b in zip(edges[:-1], edges[1:])]
    m_loss, m_row, ls, lt = O.finalize_np(O.merge_partials_np(parts), mask)
    assert abs(m_loss - loss) <= 1e-9 * max(1.0, abs(loss))
    n = mask.sum()
    gh = 0
    gw = []
    for a, b in zip(edges[:-1], edges[1:]):
        dh, dw = O.range_grads_np(h_s, h_t, W[a:b], ls, lt, mask, n, T)
        gh = gh + dh
        gw.append(dw)
    np.testing.assert_allclose(gh, dH, rtol=1e-8, atol=1e-12)
    np.testing.assert_allclose(np.concatenate(gw), dW, rtol=1e-8, atol=1e-12)


@pytest.mark.parametrize("seed,T", [(1, 1.0), (2, 2.0), (3, 0.5)])
def test_closed_form_gradients_match_finite_differences(seed, T):
    """The closed-form dH_s and dW (soft-target CE rule, teacher detached) are the derivatives
    of the closed-form loss: central differences in float64."""
    h_s, h_t, W, mask = _problem(5, 8, 11, 0.7, seed)
    mask[0] = True
    loss, dH, dW, *_ = O.aligned_kl_loss_np(h_s, h_t, W, mask, T)
    eps = 1e-6

    # the teacher is detached (train.py:183): its distribution p comes from the unperturbed W,
    # and only the student's logits h_s w^T move
    zt = h_t @ W.T / T
    p = np.exp(zt - zt.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)

    def f(hs, w):
        zs = hs @ w.T / T
        ls = zs.max(axis=1) + np.log(np.exp(zs - zs.max(axis=1, keepdims=True)).sum(axis=1))
        kl = (p * (zt - zs)).sum(axis=1) + ls - (zt * p).sum(axis=1) + (p * np.log(p)).sum(axis=1)
        return float((kl * mask).sum() / mask.sum())

    assert abs(f(h_s, W) - loss) <= 1e-12 * max(1.0, abs(loss))
    for (i, j) in [(0, 0), (1, 3), (4, 7), (2, 5)]:
        a, b = h_s.copy(), h_s.copy()
        a[i, j] += eps
        b[i, j] -= eps
        assert abs((f(a, W) - f(b, W)) / (2 * eps) - dH[i, j]) <= 1e-7 + 1e-5 * abs(dH[i, j])
    for (v, j) in [(0, 0), (3, 2), (10, 7), (6, 4)]:
        a, b = W.copy(), W.copy()
        a[v, j] += eps
        b[v, j] -= eps
        assert abs((f(h_s, a) - f(h_s, b)) / (2 * eps) - dW[v, j]) <= 1e-7 + 1e-5 * abs(dW[v, j])


def test_identical_views_give_zero_and_kl_is_nonnegative():
    """KL(p || p) = 0 with zero gradients; KL >= 0 row by row (float64)."""
    h_s, h_t, W, mask = _problem(16, 16, 50, 1.0, 7)
    loss, dH, dW, row_kl, *_ = O.aligned_kl_loss_np(h_s, h_s, W, mask, 1.3)
    assert abs(loss) < 1e-12 and np.abs(dH).max() < 1e-12 and np.abs(dW).max() < 1e-12
    loss, _, _, row_kl, *_ = O.aligned_kl_loss_np(h_s, h_t, W, mask, 1.3)
    assert (row_kl >= -1e-12).all() and loss > 0

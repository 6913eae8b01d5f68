"""Pin the sampler oracle against the reference's ``sample_token`` (generate.py:40-78).

The fixture ``tests/golden/sample_token.npz`` comes from running the reference's own
``generate.sample_token``; ``tests/golden/make_golden_sample.py`` is the generator.
The greedy tokens must match exactly (including first-index tie-breaking on exact
integer ties); the probabilities at T = 0.7 to fp32 rounding.  The Gumbel-max keys the
fused sampler uses are checked for the distribution they draw from.
"""
import math

import numpy as np

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN


def load():
    return dict(np.load(GOLDEN / "sample_token.npz"))


def test_greedy_matches_reference():
    g = load()
    tok, logit, lse, _ = O.lm_head_sample_np(g["h"], g["weight"], 0.0)
    np.testing.assert_array_equal(tok, g["greedy"])
    ref_tok, probs = O.sample_token_np(g["h"].astype(np.float64) @ g["weight"].astype(np.float64).T, 0.0)
    assert probs is None
    np.testing.assert_array_equal(ref_tok, g["greedy"])


def test_greedy_exact_ties_keep_first_index():
    g = load()
    tok, _, _, keys = O.lm_head_sample_np(g["h_int"], g["weight_int"], 0.0)
    np.testing.assert_array_equal(tok, g["greedy_int"])
    # the fixture really holds ties: duplicated weight rows 20..39 equal rows 0..19
    assert np.all(tok < 20)


def test_probabilities_match_reference():
    g = load()
    T = 0.7
    z = g["h"].astype(np.float64) @ g["weight"].astype(np.float64).T
    _, probs = O.sample_token_np(z, T)
    np.testing.assert_allclose(probs, g["probs_t07"], rtol=2e-5, atol=1e-9)
    # the fused op's outputs (token logit, lse) give p(token) = exp(z_tok / T - lse)
    tok, logit, lse, _ = O.lm_head_sample_np(g["h"], g["weight"], T, seed=5)
    p_tok = np.exp(logit / T - lse)
    np.testing.assert_allclose(p_tok, g["probs_t07"][np.arange(len(tok)), tok], rtol=2e-5)


def test_hash_and_variate_ranges():
    x = O.sample_hash_np(123, np.arange(64), np.arange(1000))
    assert x.dtype == np.uint32 and x.shape == (64, 1000)
    assert len(np.unique(x)) > 0.999 * x.size
    bits = np.unpackbits(x.view(np.uint8)).mean()
    assert abs(bits - 0.5) < 0.002
    E = O.exp_variate_log2_np(x) * math.log(2.0)     # natural units: Exp(1)
    assert E.min() > 0 and np.isfinite(E).all()
    assert abs(E.mean() - 1.0) < 0.01 and abs(E.var() - 1.0) < 0.03
    # the seed's high half matters
    assert not np.array_equal(x, O.sample_hash_np(123 + (1 << 32), np.arange(64), np.arange(1000)))


def test_gumbel_max_draws_from_softmax():
    """Rows sharing one logit vector but not the noise: token frequencies follow
    softmax(z / T) (Pearson chi-square over 24 columns)."""
    rng = np.random.default_rng(0)
    V, n, T = 24, 40000, 0.8
    z = rng.normal(size=V) * 1.5
    keys = O.sample_keys_np(np.broadcast_to(z, (n, V)), T, seed=99)
    tok = np.argmax(keys, axis=-1)
    _, p = O.sample_token_np(z[None], T)
    expected = p[0] * n
    observed = np.bincount(tok, minlength=V)
    chi2 = float(((observed - expected) ** 2 / expected).sum())
    assert chi2 < 60.0, chi2          # 23 degrees of freedom: p < 1e-4 beyond 60


FILTERS = {"k20": (0.7, 20, 1.0), "p09": (1.0, 0, 0.9), "k50p08": (0.8, 50, 0.8), "p05": (0.5, 0, 0.5),
           "k1": (1.0, 1, 1.0)}


def test_filtered_probabilities_match_reference():
    """top-k / top-p (generate.py:55-75): the oracle's filtered distribution equals the
    reference's own ``sample_token`` probabilities on the fixture, support and values."""
    g = load()
    z = g["h"].astype(np.float64) @ g["weight"].astype(np.float64).T
    for name, (T, k, p) in FILTERS.items():
        probs, kept = O.filtered_probs_np(z, T, k, p)
        ref = g[f"probs_{name}"]
        np.testing.assert_array_equal(kept, ref > 0, err_msg=name)
        np.testing.assert_allclose(probs, ref, rtol=2e-5, atol=1e-9, err_msg=name)
    assert (g["probs_k1"] > 0).sum(axis=1).max() == 1          # top-1 keeps one entry per row


def test_filtered_gumbel_keys_draw_from_filtered_softmax():
    """Gumbel-max over the kept entries draws from the filtered distribution (chi-square)."""
    rng = np.random.default_rng(3)
    V, n, T, k, p = 40, 60000, 0.9, 12, 0.85
    z = rng.normal(size=V) * 1.5
    keys = O.filtered_keys_np(np.broadcast_to(z, (n, V)), T, seed=7, top_k=k, top_p=p)
    tok = np.argmax(keys, axis=-1)
    probs, kept = O.filtered_probs_np(z[None], T, k, p)
    assert kept[0, tok].all()
    support = np.flatnonzero(kept[0])
    expected = probs[0, support] * n
    observed = np.bincount(tok, minlength=V)[support]
    chi2 = float(((observed - expected) ** 2 / expected).sum())
    assert chi2 < 3.0 * len(support) + 30.0, chi2

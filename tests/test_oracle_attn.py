"""Pin the block-diffusion attention oracle against the reference's flex-attention path.

Fixture ``tests/golden/attn_block.npz`` (generator ``make_golden_attn.py``): the
reference's ``fused_flex_attention`` with its block mask and causal-limit score_mod
(``model.py:45-96``, ``model.py:435-446``), GQA, per-position limits, -1 and past-the-end
limits.
"""
import numpy as np

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN


def test_block_attention_oracle_matches_reference_flex():
    g = dict(np.load(GOLDEN / "attn_block.npz"))
    out, lse = O.block_attention_np(g["q"], g["k_self"], g["v_self"], g["k_ar"], g["v_ar"], g["limits"], int(g["K"]))
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(lse, g["lse"], rtol=1e-5, atol=2e-5)


def test_oracle_limits_clip_and_self_keys():
    rng = np.random.default_rng(0)
    B, H, Hkv, K, Ld, D, AL = 1, 2, 1, 4, 8, 64, 10
    q, ks, vs = (rng.normal(size=s) for s in [(B, H, Ld, D), (B, Hkv, Ld, D), (B, Hkv, Ld, D)])
    ka, va = rng.normal(size=(B, Hkv, AL, D)), rng.normal(size=(B, Hkv, AL, D))
    lim = np.array([[-1] * 4 + [99] * 4])
    out, _ = O.block_attention_np(q, ks, vs, ka, va, lim, K)
    # block 0 with no AR keys: plain softmax attention over its own 4 keys
    s = q[0, 0, :4] @ ks[0, 0, :4].T / 8.0
    p = np.exp(s - s.max(1, keepdims=True))
    np.testing.assert_allclose(out[0, 0, :4], (p / p.sum(1, keepdims=True)) @ vs[0, 0, :4], rtol=1e-12)
    # a limit past the cache end sees the whole cache
    out2, _ = O.block_attention_np(q, ks, vs, ka, va, np.array([[-1] * 4 + [AL - 1] * 4]), K)
    np.testing.assert_allclose(out, out2, rtol=1e-12)


def test_block_attention_backward_oracle_matches_reference_mask():
    """The closed-form backward against gradients of the reference's attention (its own block
    mask and causal-limit rule, a dense float64 restatement whose forward the generator
    checked against the reference's flex-attention output)."""
    g = dict(np.load(GOLDEN / "attn_block_bwd.npz"))
    args = (g["q"], g["k_self"], g["v_self"], g["k_ar"], g["v_ar"], g["limits"], int(g["K"]))
    out, lse = O.block_attention_np(*args)
    np.testing.assert_allclose(out, g["out"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, g["lse"], rtol=1e-10, atol=1e-12)
    dq, dks, dvs = O.block_attention_bwd_np(*args, g["d_out"])
    for ours, ref in ((dq, g["dq"]), (dks, g["dk_self"]), (dvs, g["dv_self"])):
        np.testing.assert_allclose(ours, ref, rtol=1e-9, atol=1e-11)


def test_block_attention_backward_matches_finite_differences():
    """The closed-form backward is the derivative of the forward (float64 central differences
    of sum(out * d_out)) for queries and the blocks' own keys and values, with GQA and limits
    from none to past the cache end."""
    rng = np.random.default_rng(3)
    B, H, Hkv, K, Ld, D, AL = 1, 4, 2, 2, 6, 8, 5
    q = rng.normal(size=(B, H, Ld, D))
    ks, vs = rng.normal(size=(B, Hkv, Ld, D)), rng.normal(size=(B, Hkv, Ld, D))
    ka, va = rng.normal(size=(B, Hkv, AL, D)), rng.normal(size=(B, Hkv, AL, D))
    lim = np.array([[-1, 0, 2, 3, 4, 99]])
    d_out = rng.normal(size=(B, H, Ld, D))
    dq, dks, dvs = O.block_attention_bwd_np(q, ks, vs, ka, va, lim, K, d_out)
    eps = 1e-6

    def f(q_, ks_, vs_):
        return float((O.block_attention_np(q_, ks_, vs_, ka, va, lim, K)[0] * d_out).sum())

    for which, grad in (("q", dq), ("ks", dks), ("vs", dvs)):
        for idx in [(0, 0, 0, 0), (0, 1, 3, 5), (0, 1, 5, 7), (0, 0, 2, 1)]:
            args = {"q": q, "ks": ks, "vs": vs}
            a = {k: v.copy() for k, v in args.items()}
            b = {k: v.copy() for k, v in args.items()}
            a[which][idx] += eps
            b[which][idx] -= eps
            fd = (f(a["q"], a["ks"], a["vs"]) - f(b["q"], b["ks"], b["vs"])) / (2 * eps)
            assert abs(fd - grad[idx]) <= 1e-7 + 1e-6 * abs(grad[idx]), (which, idx, fd, grad[idx])

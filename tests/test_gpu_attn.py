"""Block-diffusion attention on the GPU against the reference's flex output and the oracle.

Tolerances: the kernel forms P in bf16 for the P V product and writes bf16 output, so the
output is compared at 3e-2 absolute (values are O(1)) with cosine >= 0.9999 against the
float64 oracle on the same bf16 inputs; the log-sum-exp (fp32 scores) at 2e-3.
"""
import math

import numpy as np
import pytest
import torch

from oracle import klgemm_oracle as O
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

OUT_ATOL = 3e-2
LSE_ATOL = 2e-3


def _dev():
    return torch.device("cuda:0")


def _check(out, lse, ref_out, ref_lse):
    from orthrus_training_test_b200 import _lib
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    err = np.abs(o - ref_out).max()
    cos = float((o * ref_out).sum() / (np.linalg.norm(o) * np.linalg.norm(ref_out)))
    assert err <= OUT_ATOL and cos >= 0.9999, (err, cos)
    if lse is not None:
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=0, atol=LSE_ATOL)


def _problem(B, H, Hkv, Ld, AL, seed, cache_len=None):
    g = torch.Generator().manual_seed(seed)
    bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)
    q, ks, vs = bf(B, H, Ld, 64), bf(B, Hkv, Ld, 64), bf(B, Hkv, Ld, 64)
    n = cache_len or AL
    ka, va = bf(B, Hkv, n, 64), bf(B, Hkv, n, 64)
    return q, ks, vs, ka, va


def test_matches_reference_flex_golden():
    from orthrus_training_test_b200.attention import block_attention
    g = dict(np.load(GOLDEN / "attn_block.npz"))
    t = lambda k: torch.tensor(g[k]).to(torch.bfloat16).to(_dev())
    out, lse = block_attention(t("q"), t("k_self"), t("v_self"), t("k_ar"), t("v_ar"),
                               torch.tensor(g["limits"]).to(_dev()), int(g["K"]), want_lse=True)
    _check(out, lse, g["out"], g["lse"])


@pytest.mark.parametrize("B,H,Hkv,K,Ld,AL,kind", [
    (1, 9, 3, 32, 32, 2047, "decode"),        # one block, the AR key range split over CTAs
    (2, 9, 3, 32, 256, 1000, "anchored"),     # training-like: each block sees the AR prefix before it
    (1, 6, 2, 64, 128, 500, "random"),        # K = 64: one query head per unit
    (1, 4, 4, 128, 256, 129, "random"),       # K = 128, no GQA, a last AR tile with one key
    (2, 6, 2, 16, 64, 300, "random"),
    (4, 9, 3, 32, 1024, 500, "anchored"),     # >= 2 units per SM: one split, output written by the kernel
])
def test_matches_oracle(B, H, Hkv, K, Ld, AL, kind):
    from orthrus_training_test_b200.attention import block_attention
    q, ks, vs, ka, va = _problem(B, H, Hkv, Ld, AL, seed=B + H + K + Ld + AL)
    g = torch.Generator().manual_seed(1)
    if kind == "decode":
        lim = torch.full((B, Ld), AL - 1)
    elif kind == "anchored":
        anchors = torch.randint(0, AL, (B, Ld // K), generator=g).sort(dim=1).values
        lim = (anchors - 1).repeat_interleave(K, dim=1)
    else:
        lim = torch.randint(-3, AL + 5, (B, Ld), generator=g)
    out, lse = block_attention(q.to(_dev()), ks.to(_dev()), vs.to(_dev()), ka.to(_dev()), va.to(_dev()),
                               lim.to(_dev()), K, want_lse=True)
    ro, rl = O.block_attention_np(q.float().numpy(), ks.float().numpy(), vs.float().numpy(), ka.float().numpy(),
                                  va.float().numpy(), lim.numpy(), K)
    _check(out, lse, ro, rl)


def test_cache_view_ignores_rows_past_ar_len():
    """k_ar / v_ar as the first ar_len rows of a longer cache whose other rows hold NaN."""
    from orthrus_training_test_b200.attention import block_attention
    B, H, Hkv, K, Ld, AL, CL = 2, 6, 2, 32, 64, 333, 600
    q, ks, vs, ka, va = _problem(B, H, Hkv, Ld, AL, seed=5, cache_len=CL)
    ka[:, :, AL:] = float("nan")
    va[:, :, AL:] = float("nan")
    lim = torch.full((B, Ld), 10_000)
    kd, vd = ka.to(_dev()), va.to(_dev())
    out = block_attention(q.to(_dev()), ks.to(_dev()), vs.to(_dev()), kd[:, :, :AL], vd[:, :, :AL], lim.to(_dev()), K)
    ro, _ = O.block_attention_np(q.float().numpy(), ks.float().numpy(), vs.float().numpy(),
                                 ka[:, :, :AL].float().numpy(), va[:, :, :AL].float().numpy(), lim.numpy(), K)
    _check(out, None, ro, None)


def test_reference_triton_api_and_fp32_inputs():
    from orthrus_training_test_b200.attention import triton_block_attention
    B, H, Hkv, K, NB, AL = 1, 9, 3, 32, 2, 700
    Ld = NB * K
    q, ks, vs, ka, va = _problem(B, H, Hkv, Ld, AL, seed=9)
    lim = torch.tensor([[200] * K + [650] * K])
    d = _dev()
    out = triton_block_attention(q.float().view(B * H, Ld, 64).to(d), ks.float().view(B * Hkv, Ld, 64).to(d),
                                 vs.float().view(B * Hkv, Ld, 64).to(d), ka.float().view(B * Hkv, AL, 64).to(d),
                                 va.float().view(B * Hkv, AL, 64).to(d), lim.to(d), B, H, Hkv, H // Hkv, 4, NB, K, AL,
                                 64)
    assert out.shape == (B * H, Ld, 64) and out.dtype == torch.float32
    ro, _ = O.block_attention_np(q.float().numpy(), ks.float().numpy(), vs.float().numpy(), ka.float().numpy(),
                                 va.float().numpy(), lim.numpy(), K)
    _check(out.view(B, H, Ld, 64), None, ro, None)


# ----------------------------------------------------------------- backward
# P and dS pass through bf16 shared-memory tiles (as the forward's P does), so the gradients
# are compared with float64 at 3e-2 normalised max error and cosine >= 0.9995.
BWD_MAX_REL = 3e-2
BWD_COS = 0.9995


def _bwd_close(ours, ref, what):
    mr, cos = O.grad_metrics(ours, ref)
    assert mr <= BWD_MAX_REL and cos >= BWD_COS, f"{what}: max-rel {mr:.3e} cos {cos:.6f}"


def _run_bwd(q, ks, vs, ka, va, lim, K, d_out):
    from orthrus_training_test_b200 import _lib
    from orthrus_training_test_b200.attention import block_attention
    dev = torch.device("cuda:0")
    qd = q.to(dev, torch.bfloat16).requires_grad_(True)
    ksd = ks.to(dev, torch.bfloat16).requires_grad_(True)
    vsd = vs.to(dev, torch.bfloat16).requires_grad_(True)
    out = block_attention(qd, ksd, vsd, ka.to(dev, torch.bfloat16), va.to(dev, torch.bfloat16), lim.to(dev), K)
    out.backward(d_out.to(dev, torch.bfloat16))
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0
    return out, qd.grad.double().cpu().numpy(), ksd.grad.double().cpu().numpy(), vsd.grad.double().cpu().numpy()


def test_backward_matches_reference_golden():
    """dQ, dK_self, dV_self against gradients of the reference's attention (fixture from its
    block mask and causal-limit rule; GQA with 3 query heads per KV head, per-position limits,
    -1 and past-the-end limits)."""
    g = dict(np.load(GOLDEN / "attn_block_bwd.npz"))
    t = lambda k: torch.tensor(g[k])
    out, dq, dks, dvs = _run_bwd(t("q"), t("k_self"), t("v_self"), t("k_ar"), t("v_ar"), t("limits"), int(g["K"]),
                                 t("d_out"))
    assert float((out.float().cpu() - t("out")).abs().max()) <= 3e-2
    _bwd_close(dq, g["dq"], "dq")
    _bwd_close(dks, g["dk_self"], "dk_self")
    _bwd_close(dvs, g["dv_self"], "dv_self")


@pytest.mark.parametrize("B,H,Hkv,K,NB,AL", [(1, 9, 3, 32, 8, 600), (2, 16, 2, 32, 3, 300), (1, 4, 4, 64, 2, 129),
                                             (1, 3, 1, 128, 2, 256)])
def test_backward_against_oracle(B, H, Hkv, K, NB, AL):
    """SmolLM2-135M heads (9 / 3, K = 32), eight query heads per KV head (two head groups add
    into the same dK / dV), no GQA with K = 64, and one head with K = 128; limits vary per
    position, including -1 and the cache end."""
    g = torch.Generator().manual_seed(B * 100 + H + K)
    Ld = NB * K
    q = torch.randn(B, H, Ld, 64, generator=g).to(torch.bfloat16).float()
    ks, vs = (torch.randn(B, Hkv, Ld, 64, generator=g).to(torch.bfloat16).float() for _ in range(2))
    ka, va = (torch.randn(B, Hkv, AL, 64, generator=g).to(torch.bfloat16).float() for _ in range(2))
    d_out = torch.randn(B, H, Ld, 64, generator=g).to(torch.bfloat16).float()
    lim = torch.randint(-1, AL + 5, (B, Ld), generator=g)
    lim[0, :K] = -1
    _, dq, dks, dvs = _run_bwd(q, ks, vs, ka, va, lim, K, d_out)
    rq, rks, rvs = O.block_attention_bwd_np(q.numpy(), ks.numpy(), vs.numpy(), ka.numpy(), va.numpy(), lim.numpy(),
                                            K, d_out.numpy())
    _bwd_close(dq, rq, "dq")
    _bwd_close(dks, rks, "dk_self")
    _bwd_close(dvs, rvs, "dv_self")

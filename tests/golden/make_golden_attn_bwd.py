"""Golden gradients of the block-diffusion attention, pinned to the reference's mask.

flex_attention has no CPU backward, so the gradients come from a dense restatement of the
reference's attention: the reference's own block mask (the ``mask_mod`` of
``build_dual_pass_block_mask``, ``model.py:64-96``, materialised with ``create_mask``) and its
causal-limit rule (``model.py:435-446``: an AR key ``kv`` is hidden from query ``q`` when
``kv > causal_limit[b, q]``), GQA by repeating the KV heads, scale 1/sqrt(64), softmax and
autograd in float64.  The generator checks that this dense forward reproduces the reference's
``fused_flex_attention`` output (``model.py:45-58``) before it writes anything.  The fixture
holds the inputs, an upstream gradient dO, the forward output and log-sum-exp, and dQ,
dK_self, dV_self (the trainable side: the diffusion heads' queries, keys and values; the AR
cache comes from the frozen backbone).

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden_attn_bwd.py [/path/to/reference]
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
REF = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
OUT = Path(__file__).resolve().parent


def main():
    sys.path.insert(0, REF)
    import warnings

    import torch
    import model as M  # reference module
    from torch.nn.attention.flex_attention import create_mask

    warnings.filterwarnings("ignore")
    g = torch.Generator().manual_seed(29)
    B, H, Hkv, K, NB, D, AL = 2, 6, 2, 16, 3, 64, 200
    Ld = NB * K
    bf = lambda t: t.to(torch.bfloat16).float()
    q = bf(torch.randn(B, H, Ld, D, generator=g))
    k_self = bf(torch.randn(B, Hkv, Ld, D, generator=g))
    v_self = bf(torch.randn(B, Hkv, Ld, D, generator=g))
    k_ar = bf(torch.randn(B, Hkv, AL, D, generator=g))
    v_ar = bf(torch.randn(B, Hkv, AL, D, generator=g))
    d_out = bf(torch.randn(B, H, Ld, D, generator=g))
    limits = torch.tensor([[30] * K + list(range(90, 90 + K)) + [199] * K,
                           [-1] * K + [120] * (K // 2) + [5] * (K // 2) + [250] * K], dtype=torch.long)
    bmask = M.build_dual_pass_block_mask(B, H, Ld, AL, K, "cpu")

    def hide_past_limit(score, b, h, q_idx, kv_idx):
        return torch.where((kv_idx < AL) & (kv_idx > limits[b, q_idx]), float("-inf"), score)

    k_full = torch.cat([k_ar, k_self], dim=2)
    v_full = torch.cat([v_ar, v_self], dim=2)
    ref_out = M.fused_flex_attention(q, k_full, v_full, mask=bmask, score_mod=hide_past_limit)

    # dense restatement with the reference's mask_mod and limit rule, float64 autograd
    allowed = create_mask(bmask.mask_mod, B, H, Ld, AL + Ld, device="cpu")           # [B, H, Ld, AL + Ld]
    kv = torch.arange(AL + Ld)
    hidden = (kv[None, None, :] < AL) & (kv[None, None, :] > limits[:, :, None])       # [B, Ld, AL + Ld]
    allowed = allowed & ~hidden[:, None]
    qd = q.double().requires_grad_(True)
    ksd = k_self.double().requires_grad_(True)
    vsd = v_self.double().requires_grad_(True)
    kf = torch.cat([k_ar.double(), ksd], dim=2).repeat_interleave(H // Hkv, dim=1)
    vf = torch.cat([v_ar.double(), vsd], dim=2).repeat_interleave(H // Hkv, dim=1)
    s = qd @ kf.transpose(-1, -2) / math.sqrt(D)
    s = s.masked_fill(~allowed, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    out = torch.softmax(s, dim=-1) @ vf
    assert torch.allclose(out.float(), ref_out, atol=2e-5), float((out.float() - ref_out).abs().max())
    (out * d_out.double()).sum().backward()
    np.savez_compressed(OUT / "attn_block_bwd.npz", q=q.numpy(), k_self=k_self.numpy(), v_self=v_self.numpy(),
                        k_ar=k_ar.numpy(), v_ar=v_ar.numpy(), limits=limits.numpy(), K=np.int64(K),
                        d_out=d_out.numpy(), out=out.detach().numpy(), lse=lse.detach().numpy(),
                        dq=qd.grad.numpy(), dk_self=ksd.grad.numpy(), dv_self=vsd.grad.numpy())
    print("attn_block_bwd:", float(qd.grad.abs().max()), float(ksd.grad.abs().max()), float(vsd.grad.abs().max()))


if __name__ == "__main__":
    main()

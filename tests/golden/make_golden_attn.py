"""Golden vectors for the block-diffusion attention from the reference's flex-attention path.

Runs the reference's ``fused_flex_attention`` (``model.py:45-58``) with its block mask
``build_dual_pass_block_mask`` (``model.py:64-96``) and the causal-limit score_mod that
``forward_diffusion`` builds (``model.py:435-446``: an AR key ``kv`` is hidden from query
``q`` when ``kv > causal_limit[b, q]``), eagerly on the CPU, with GQA (3 query heads per KV
head), per-position limits that vary inside a block, limits of -1 and past the cache end.
Inputs are bf16-representable fp32; the fixture stores them with the output and the
log-sum-exp (flex_attention's ``return_lse``).

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden_attn.py [/path/to/reference]
"""
from __future__ import annotations

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
    from torch.nn.attention.flex_attention import flex_attention

    warnings.filterwarnings("ignore")
    g = torch.Generator().manual_seed(23)
    B, H, Hkv, K, NB, D, AL = 2, 6, 2, 16, 3, 64, 300
    Ld = NB * K
    bf = lambda t: t.to(torch.bfloat16).float()
    q = bf(torch.randn(B, H, Ld, D, generator=g))
    k_self = bf(torch.randn(B, Hkv, Ld, D, generator=g))
    v_self = bf(torch.randn(B, Hkv, Ld, D, generator=g))
    k_ar = bf(torch.randn(B, Hkv, AL, D, generator=g))
    v_ar = bf(torch.randn(B, Hkv, AL, D, generator=g))
    limits = torch.tensor([[40] * K + list(range(100, 100 + K)) + [299] * K,
                           [-1] * K + [130] * (K // 2) + [7] * (K // 2) + [400] * K], dtype=torch.long)
    mask = M.build_dual_pass_block_mask(B, H, Ld, AL, K, "cpu")

    def hide_past_limit(score, b, h, q_idx, kv_idx):
        return torch.where((kv_idx < AL) & (kv_idx > limits[b, q_idx]), float("-inf"), score)

    k_full = torch.cat([k_ar, k_self], dim=2)
    v_full = torch.cat([v_ar, v_self], dim=2)
    out = M.fused_flex_attention(q, k_full, v_full, mask=mask, score_mod=hide_past_limit)
    kw = {"sparse_block_size": (int(mask.BLOCK_SIZE[0]), int(mask.BLOCK_SIZE[1]))}
    out2, lse = flex_attention(q, k_full, v_full, block_mask=mask, score_mod=hide_past_limit, enable_gqa=True,
                               kernel_options=kw, return_lse=True)
    assert torch.allclose(out, out2)
    np.savez_compressed(OUT / "attn_block.npz", q=q.numpy(), k_self=k_self.numpy(), v_self=v_self.numpy(),
                        k_ar=k_ar.numpy(), v_ar=v_ar.numpy(), limits=limits.numpy(), K=np.int64(K),
                        out=out.numpy(), lse=lse.numpy())
    print("attn_block:", tuple(out.shape), float(out.abs().max()))


if __name__ == "__main__":
    main()

"""Golden vectors for the fused final-RMSNorm prologue (pre-norm inputs).

The reference applies the backbone's final norm (``model.py:493``, ``self.norm`` = the base
model's ``LlamaRMSNorm`` from transformers, weight frozen by ``model.py:323-324``) before the
lm_head, then ``train.compute_kl_loss`` (``train.py:142-195``).  This script runs both from
the reference checkout and transformers (5.5.0 here) on small seeded inputs:

* ``norm_bf16``: bf16 rows through ``LlamaRMSNorm(eps=1e-5)`` with a bf16 weight -- the
  norm's output in a bf16 model, bit for bit.
* ``norm_loss``: fp32 pre-norm rows -> ``LlamaRMSNorm`` (fp32) -> ``compute_kl_loss`` on the
  aligned row layout; stores the loss and the gradient of the pre-norm student rows.

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden_norm.py [/path/to/reference]
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
REF = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
OUT = Path(__file__).resolve().parent
EPS = 1e-5


def main():
    sys.path.insert(0, REF)
    import torch
    import train  # reference module
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    g = torch.Generator().manual_seed(17)

    # 1) bf16 norm output
    N, H = 64, 576
    x = (torch.randn(N, H, generator=g) * 3.0).to(torch.bfloat16)
    x[5] *= 40.0                                     # a row with large activations
    gamma = (1.0 + 0.3 * torch.randn(H, generator=g)).to(torch.bfloat16)
    norm = LlamaRMSNorm(H, eps=EPS)
    norm.weight.data = gamma.clone()
    with torch.no_grad():
        y = norm(x)
    assert y.dtype == torch.bfloat16
    np.savez_compressed(OUT / "norm_bf16.npz", x=x.float().numpy(), gamma=gamma.float().numpy(),
                        y=y.float().numpy(), eps=np.float64(EPS))

    # 2) loss through the norm, fp32, aligned rows: student rows blk*K + k (k >= 1), teacher
    #    rows anchor + k - 1 with anchors K - 1 apart (contiguous teacher positions)
    B, B_blocks, K, H2, V = 1, 4, 8, 64, 300
    Nr = B_blocks * (K - 1)
    bf = lambda t: t.to(torch.bfloat16).float()
    h_s = bf(torch.randn(Nr, H2, generator=g) * 2.0)
    h_t = bf(torch.randn(Nr, H2, generator=g) * 2.0)
    gam = bf(1.0 + 0.2 * torch.randn(H2, generator=g))
    W = bf(torch.randn(V, H2, generator=g) * 0.1)
    mask = torch.rand(Nr, generator=g) < 0.7
    diff = torch.randn(B, B_blocks * K, H2, generator=g)
    ar = torch.empty(B, B_blocks * (K - 1), H2)
    tgt = torch.full((B, B_blocks * K), 7, dtype=torch.long)
    anchors = (torch.arange(B_blocks) * (K - 1)).unsqueeze(0)
    for blk in range(B_blocks):
        for k in range(1, K):
            r = blk * (K - 1) + (k - 1)
            diff[0, blk * K + k] = h_s[r]
            ar[0, r] = h_t[r]
            if not mask[r]:
                tgt[0, blk * K + k] = 0
    norm2 = LlamaRMSNorm(H2, eps=EPS)
    norm2.weight.data = gam.clone()
    head = torch.nn.Linear(H2, V, bias=False)
    head.weight.data = W.clone()
    diff = diff.requires_grad_(True)
    loss = train.compute_kl_loss(norm2(diff), norm2(ar).detach(), head, anchors, K, tgt, 0)
    loss.backward()
    rows = [blk * K + k for blk in range(B_blocks) for k in range(1, K)]
    g_rows = diff.grad[0, rows].numpy()
    np.savez_compressed(OUT / "norm_loss.npz", h_s=h_s.numpy(), h_t=h_t.numpy(), gamma=gam.numpy(),
                        weight=W.numpy(), mask=mask.numpy(), eps=np.float64(EPS), loss=np.float64(loss.item()),
                        grad_h_s=g_rows)
    print(f"norm_bf16: {N}x{H}; norm_loss: loss={loss.item():.6f}")


if __name__ == "__main__":
    main()

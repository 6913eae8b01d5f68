"""Generate golden vectors by running the reference's own loss.

Runs ``train.compute_kl_loss`` from the reference checkout (``train.py:142-195``,
with ``_kl_chunk_body`` at ``train.py:198-210``) on small seeded inputs and
stores inputs and outputs (loss, grad of the student hidden states, grad of
the lm_head weight) as ``.npz`` fixtures beside this script.

Only runs where the reference checkout exists (the build container); the
fixtures it writes are committed and are what the tests read.

    TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden.py [/path/to/reference]

``TORCHDYNAMO_DISABLE=1`` is needed because ``_kl_chunk_body`` is wrapped in
``torch.compile`` (train.py:198), whose CPU backend does not build in this
container; with it set the function runs eagerly, which is its defined
semantics.  Importing the reference turns TF32 and "medium" matmul precision
on (train.py:47-50); they are reset to strict fp32 before anything runs.
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
    import torch
    import train  # reference module

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    F = torch.nn.functional

    class Head(torch.nn.Module):
        """lm_head with optional temperature: ``linear(x, W) / T``."""

        def __init__(self, W, T):
            super().__init__()
            self.weight = torch.nn.Parameter(W.clone())
            self.T = T

        def forward(self, x):
            z = F.linear(x, self.weight)
            return z if self.T == 1.0 else z / self.T

    def aligned_layout(h_s, h_t, mask, B, B_blocks, K, pad, gen):
        """Embeds aligned rows into compute_kl_loss's gather layout.

        Anchors are spaced K-1 apart so teacher rows ``anchor + k - 1`` are the
        contiguous positions ``blk*(K-1) + k - 1``; student rows are
        ``blk*K + k`` (k >= 1).  Anchor (k = 0) rows get random values that the
        loss must ignore.
        """
        H = h_s.shape[1]
        N = B_blocks * (K - 1)
        diff = torch.randn(B, B_blocks * K, H, generator=gen)
        ar = torch.empty(B, B_blocks * (K - 1), H)
        tgt = torch.full((B, B_blocks * K), 7, dtype=torch.long)
        anchors = (torch.arange(B_blocks) * (K - 1)).unsqueeze(0).repeat(B, 1)
        for b in range(B):
            for blk in range(B_blocks):
                for k in range(1, K):
                    r = b * N + blk * (K - 1) + (k - 1)
                    diff[b, blk * K + k] = h_s[r]
                    ar[b, blk * (K - 1) + k - 1] = h_t[r]
                    if not mask[r]:
                        tgt[b, blk * K + k] = pad
        return diff, ar, anchors, tgt

    def run(name, diff, ar, anchors, K, tgt, pad, W, T, extra):
        head = Head(W, T)
        diff = diff.clone().requires_grad_(True)
        loss = train.compute_kl_loss(diff, ar, head, anchors, K, tgt, pad)
        if loss.grad_fn is not None:
            loss.backward()
            g_diff = diff.grad.numpy() if diff.grad is not None else np.zeros(diff.shape, np.float32)
            g_w = head.weight.grad.numpy() if head.weight.grad is not None else np.zeros(W.shape, np.float32)
        else:
            g_diff = np.zeros(diff.shape, np.float32)
            g_w = np.zeros(W.shape, np.float32)
        arrays = dict(diff_hidden=diff.detach().numpy(), ar_hidden=ar.numpy(),
                      anchor_positions=anchors.numpy(), target_ids=tgt.numpy(),
                      weight=W.numpy(), K=np.int64(K), pad=np.int64(pad),
                      temperature=np.float64(T), loss=np.float64(loss.item()),
                      grad_diff_hidden=g_diff, grad_weight=g_w)
        arrays.update(extra)
        np.savez_compressed(OUT / f"{name}.npz", **arrays)
        print(f"{name}: loss={loss.item():.6f}")

    pad = 0
    # aligned cases: N = B * B_blocks * (K-1) rows
    cases = [
        # name, B, B_blocks, K, H, V, T, teacher scale, mask prob, seed
        ("aligned_t1", 2, 4, 8, 64, 517, 1.0, 1.0, 0.5, 1),
        ("aligned_t2_peaky", 2, 4, 8, 64, 517, 2.0, 4.0, 0.25, 2),
        ("aligned_h128_v300", 1, 6, 9, 128, 300, 1.0, 1.0, 0.7, 3),
    ]
    for name, B, B_blocks, K, H, V, T, ts, pm, seed in cases:
        g = torch.Generator().manual_seed(seed)
        N = B * B_blocks * (K - 1)
        h_s = torch.randn(N, H, generator=g)
        h_t = torch.randn(N, H, generator=g) * ts
        W = torch.randn(V, H, generator=g) * 0.02 * (4.0 if name.endswith("peaky") else 1.0)
        mask = torch.rand(N, generator=g) < pm
        if name == "aligned_t2_peaky":
            mask[:8] = False  # fully masked rows inside a block
        diff, ar, anchors, tgt = aligned_layout(h_s, h_t, mask, B, B_blocks, K, pad, g)
        run(name, diff, ar, anchors, K, tgt, pad, W, T,
            dict(h_s=h_s.numpy(), h_t=h_t.numpy(), mask=mask.numpy()))

    # real anchor layout with clamping at the sequence end (train.py:161)
    g = torch.Generator().manual_seed(4)
    B, L, B_blocks, K, H, V = 2, 20, 3, 6, 64, 203
    diff = torch.randn(B, B_blocks * K, H, generator=g)
    ar = torch.randn(B, L, H, generator=g)
    anchors = torch.tensor([[0, 9, 17], [3, 15, 19]])
    tgt = torch.randint(1, 50, (B, B_blocks * K), generator=g)
    tgt[torch.rand(tgt.shape, generator=g) < 0.3] = pad
    W = torch.randn(V, H, generator=g) * 0.02
    run("anchors_clamp", diff, ar, anchors, K, tgt, pad, W, 1.0, {})

    # nothing valid: early return 0.0 (train.py:166-167)
    tgt0 = torch.full_like(tgt, pad)
    run("all_masked", diff, ar, anchors, K, tgt0, pad, W, 1.0, {})


if __name__ == "__main__":
    main()

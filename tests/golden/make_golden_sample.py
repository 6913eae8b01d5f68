"""Generate golden vectors for the inference sampler from the reference's ``sample_token``.

Runs ``generate.sample_token`` (reference ``generate.py:40-78``) on lm_head logits of
small seeded inputs and stores the inputs (hidden rows, lm_head weight) with its greedy
tokens (``temperature = 0``) and its probabilities at ``temperature = 0.7``.  The sampled
tokens themselves come from ``torch.multinomial``'s generator and are not stored: the
fused sampler is checked against the distribution, not the stream.

Only runs where the reference checkout exists (the build container); the fixture it
writes is committed and is what the tests read.

    python tests/golden/make_golden_sample.py [/path/to/reference]
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

REF = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
OUT = Path(__file__).resolve().parent


def main():
    sys.path.insert(0, REF)
    import torch
    import generate  # reference module

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    g = torch.Generator().manual_seed(11)
    arrays = {}

    # seeded normal rows, bf16-representable; logits in fp32 as the model computes them
    N, H, V = 24, 64, 517
    h = torch.randn(N, H, generator=g).to(torch.bfloat16).float()
    W = (torch.randn(V, H, generator=g) * 0.3).to(torch.bfloat16).float()
    z = h @ W.T
    tok, probs = generate.sample_token(z.clone(), 0.0)
    assert probs is None
    _, p07 = generate.sample_token(z.clone(), 0.7)
    arrays.update(h=h.numpy(), weight=W.numpy(), greedy=tok.numpy(), probs_t07=p07.numpy())
    # top-k / top-p (generate.py:59-73): the reference's filtered probabilities
    for name, (T, k, p) in {"k20": (0.7, 20, 1.0), "p09": (1.0, 0, 0.9), "k50p08": (0.8, 50, 0.8),
                            "p05": (0.5, 0, 0.5), "k1": (1.0, 1, 1.0)}.items():
        _, pf = generate.sample_token(z.clone(), T, k, p)
        arrays[f"probs_{name}"] = pf.numpy()

    # small integer rows and duplicated weight rows: exact ties, where argmax keeps the first
    Ni, Hi, Vi = 16, 32, 40
    hi = torch.randint(-1, 2, (Ni, Hi), generator=g).float()
    Wi = torch.randint(-1, 2, (Vi, Hi), generator=g).float()
    Wi[20:] = Wi[:20]
    zi = hi @ Wi.T
    toki, _ = generate.sample_token(zi.clone(), 0.0)
    arrays.update(h_int=hi.numpy(), weight_int=Wi.numpy(), greedy_int=toki.numpy())

    np.savez_compressed(OUT / "sample_token.npz", **arrays)
    print("sample_token:", tok[:8].tolist(), toki[:8].tolist())


if __name__ == "__main__":
    main()
